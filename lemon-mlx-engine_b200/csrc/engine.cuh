// engine.cuh -- the C++ host side of the speculative-decode path: model
// weights, KV caches, the verify / draft forward graph and the speculative
// loop.  It mirrors the reference's TokenIterator contract
// (src/common/generate.cpp:669-933, :968-1045): d0 is emitted first, then the
// accepted drafts; the next d0 is the correction / bonus token; the target
// cache is rolled back to p+acc+1.  Everything per step stays on the device
// and one step is captured as a CUDA graph.
#pragma once
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "lmx_internal.h"

namespace lmx {

// ---------------------------------------------------------------------------
// launchers of the attention / engine kernels
// ---------------------------------------------------------------------------
static int launch_attn_prep(const PrepArgs& a, cudaStream_t st) {
  const int tasks = a.R * (a.Hq + 2 * a.Hk);
  if (tasks == 0) return LMX_OK;
  return cuda_check(lmx_launch(attn_prep_kernel, dim3((tasks + 7) / 8), dim3(256), 0, st, true, a),
                    "attn_prep: launch");
}

template <int RPT>
static int launch_sdpa_t(const SdpaArgs& a, int B, cudaStream_t st) {
  static bool attr_set[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  if (!attr_set[d & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(sdpa_split_kernel<RPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kSdpaSmem),
                        "sdpa: set smem");
    if (rc) return rc;
    attr_set[d & 63] = true;
  }
  return cuda_check(lmx_launch(sdpa_split_kernel<RPT>, dim3(a.nsplit * a.tiles, a.kv.Hk, B), dim3(256),
                               kSdpaSmem, st, true, a),
                    "sdpa: launch");
}

// Cache rows from which every block (also a single decode token) takes the
// tensor-core SDPA in tensor-core mode; process-wide, lmx_set_sdpa_tc_min_cache.
// Default 1 (every block): measured on the B200 the tensor-core kernel is the
// faster one for single-token decode at every capacity tried (8 sequences,
// 16 q / 8 kv heads, 4-bit cache: 9.8 us vs 16.4 us at 130 rows, 23.2 vs
// 51.9 us at 1030, 33.1 vs 88.7 us at 1800).
static int g_sdpa_long_cache = 1;

// Tensor-core SDPA geometry (attn_mma.cuh): row tiles of 16*MT <= 64 rows,
// nsplit key splits per (sequence, KV head, tile), as many as one wave of
// resident CTAs holds (at most one per 128-key chunk of the capacity).  The
// kernel divides the chunks a block actually reaches (the cache length on
// the device) evenly over the splits, so a graph captured once stays
// balanced as the caches grow.
struct SdpaMmaPlan {
  int MT = 1, tiles = 1, nsplit = 1;
};
template <int MT, int BITS>
static int sdpa_mma_occupancy() {
  static int occ[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  if (!occ[d & 63]) {
    int n = 0;
    if (cudaFuncSetAttribute(sdpa_mma_kernel<MT, BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sdpa_mma_smem<MT, BITS>()) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, sdpa_mma_kernel<MT, BITS>, kAttnThreads,
                                                      sdpa_mma_smem<MT, BITS>()) != cudaSuccess ||
        n < 1) {
      (void)cudaGetLastError();
      n = 1;
    }
    occ[d & 63] = n;
  }
  return occ[d & 63];
}
template <int MT>
static int sdpa_mma_occupancy_t(int bits) {
  return bits == 8 ? sdpa_mma_occupancy<MT, 8>() : (bits == 4 ? sdpa_mma_occupancy<MT, 4>()
                                                               : sdpa_mma_occupancy<MT, 16>());
}
static SdpaMmaPlan sdpa_mma_plan(int B, int Hk, int rows, int cap, int bits) {
  SdpaMmaPlan p;
  const int r = rows < kAttnMmaRows ? rows : kAttnMmaRows;
  p.MT = (r + 15) / 16;
  p.tiles = (rows + 16 * p.MT - 1) / (16 * p.MT);
  const int occ = p.MT == 1 ? sdpa_mma_occupancy_t<1>(bits)
                            : (p.MT == 2 ? sdpa_mma_occupancy_t<2>(bits)
                                         : (p.MT == 3 ? sdpa_mma_occupancy_t<3>(bits) : sdpa_mma_occupancy_t<4>(bits)));
  const int chunks = (cap + kAttnChunk - 1) / kAttnChunk;
  const int base = B * Hk * p.tiles;
  p.nsplit = std::max(1, std::min(chunks, occ * device_sms() / std::max(1, base)));
  return p;
}

// Scratch (floats / counters) that covers both SDPA paths for up to Tmax
// query tokens per sequence.
static void sdpa_scratch_need(int B, int Tmax, int G, int Hk, int cap, size_t& part_floats, size_t& counters) {
  const int chunks = (cap + kSplit - 1) / kSplit;
  const size_t rows32 = (size_t)((G * Tmax + kRowTile - 1) / kRowTile) * kRowTile;
  const size_t rows64 = (size_t)((G * Tmax + kAttnMmaRows - 1) / kAttnMmaRows) * kAttnMmaRows;
  part_floats = (size_t)B * Hk * chunks * kPartStride * std::max(rows32, rows64);
  counters = (size_t)B * Hk * ((G * Tmax + kRowTile - 1) / kRowTile);
}

template <int MT, int BITS>
static int launch_sdpa_mma_tb(const SdpaArgs& a, int B, cudaStream_t st) {
  static bool attr_set[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  if (!attr_set[d & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(sdpa_mma_kernel<MT, BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sdpa_mma_smem<MT, BITS>()),
                        "sdpa_mma: set smem");
    if (rc) return rc;
    attr_set[d & 63] = true;
  }
  return cuda_check(lmx_launch(sdpa_mma_kernel<MT, BITS>, dim3(a.nsplit * a.tiles, a.kv.Hk, B), dim3(kAttnThreads),
                               sdpa_mma_smem<MT, BITS>(), st, true, a),
                    "sdpa_mma: launch");
}
template <int MT>
static int launch_sdpa_mma_t(const SdpaArgs& a, int B, cudaStream_t st) {
  if (a.kv.bits == 8) return launch_sdpa_mma_tb<MT, 8>(a, B, st);
  if (a.kv.bits == 4) return launch_sdpa_mma_tb<MT, 4>(a, B, st);
  return launch_sdpa_mma_tb<MT, 16>(a, B, st);
}

static int launch_sdpa(const SdpaArgs& a_in, int B, cudaStream_t st) {
  const int rows = (a_in.Hq / a_in.kv.Hk) * a_in.T;
  // tensor-core kernel (unless in exact mode): blocks of >= threshold query
  // rows per KV head (verify), and any block over a long cache, where its
  // bulk-copy pipeline streams the cache far faster than the canonical
  // kernel's per-split loads
  if (qmm_uses_mma(rows) || (qmm_mma_min_m() > 0 && g_sdpa_long_cache > 0 && a_in.kv.cap >= g_sdpa_long_cache)) {
    SdpaArgs a = a_in;
    const SdpaMmaPlan p = sdpa_mma_plan(B, a.kv.Hk, rows, a.kv.cap, a.kv.bits);
    a.err = device_error_word();
    a.tiles = p.tiles;
    a.nsplit = p.nsplit;
    if ((size_t)B * a.kv.Hk * p.tiles * p.nsplit * kAttnMmaRows * kPartStride > a.part_floats ||
        (size_t)B * a.kv.Hk * p.tiles > a.n_counters)
      return set_error(LMX_ERR_INVALID, "sdpa: scratch too small for the tensor-core path");
    switch (p.MT) {
      case 1: return launch_sdpa_mma_t<1>(a, B, st);
      case 2: return launch_sdpa_mma_t<2>(a, B, st);
      case 3: return launch_sdpa_mma_t<3>(a, B, st);
      default: return launch_sdpa_mma_t<4>(a, B, st);
    }
  }
  const SdpaArgs& a = a_in;
  if ((size_t)B * a.kv.Hk * a.tiles * a.nsplit * kRowTile * kPartStride > a.part_floats ||
      (size_t)B * a.kv.Hk * a.tiles > a.n_counters)
    return set_error(LMX_ERR_INVALID, "sdpa: scratch too small");
  const int half = ((rows < kRowTile ? rows : kRowTile) + 1) / 2;  // rows per thread needed
  if (half <= 1) return launch_sdpa_t<1>(a, B, st);
  if (half <= 2) return launch_sdpa_t<2>(a, B, st);
  if (half <= 3) return launch_sdpa_t<3>(a, B, st);
  if (half <= 4) return launch_sdpa_t<4>(a, B, st);
  if (half <= 5) return launch_sdpa_t<5>(a, B, st);
  if (half <= 6) return launch_sdpa_t<6>(a, B, st);
  if (half <= 8) return launch_sdpa_t<8>(a, B, st);
  if (half <= 12) return launch_sdpa_t<12>(a, B, st);
  return launch_sdpa_t<16>(a, B, st);
}

static int launch_cluster_rows(void (*kern)(const bf16_t*, int, SpecState, int, int), int rows,
                               const bf16_t* logits, int V, const SpecState& s, int i, int adv,
                               cudaStream_t st) {
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
  return cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, kern, logits, V, s, i, adv)), "draft_argmax: launch");
}

// ---------------------------------------------------------------------------
// device memory arena (setup-time allocations only)
// ---------------------------------------------------------------------------
struct DevBuf {
  void* p = nullptr;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { if (p) cudaFree(p); }
};

struct Arena {
  std::vector<std::unique_ptr<DevBuf>> bufs;
  template <typename T>
  int alloc(T** out, size_t count, bool zero = true) {
    auto b = std::make_unique<DevBuf>();
    const size_t bytes = count * sizeof(T) > 0 ? count * sizeof(T) : 16;
    if (cudaMalloc(&b->p, bytes) != cudaSuccess) {
      cudaGetLastError();
      return set_error(LMX_ERR_OOM, "cudaMalloc(%zu) failed", bytes);
    }
    if (zero && cudaMemset(b->p, 0, bytes) != cudaSuccess) return cuda_check(cudaGetLastError(), "memset");
    *out = (T*)b->p;
    bufs.push_back(std::move(b));
    return LMX_OK;
  }
};

// ---------------------------------------------------------------------------
// tensor-parallel communicator: this rank's IPC-exported block (two partial
// slots, the argmax pairs, the arrival flags) and the peers' blocks opened
// through their handles.  Layout and protocol: tp.cuh.
// ---------------------------------------------------------------------------
struct TpComm {
  int n = 1, rank = 0, max_rows = 0, max_hidden = 0;
  void* block = nullptr;  // local, from cudaMalloc (exportable)
  size_t block_bytes = 0;
  uint32_t* epoch = nullptr;
  void* peer[kTpMaxRanks] = {};      // opened through IPC handles (closed here)
  bool attached[kTpMaxRanks] = {};   // attached by pointer (the caller's mapping)
  bool opened = false;
  int sel = 0;  // partial slot of the next exchange: alternates over every exchange on the comm
  TpPeers t;
  ~TpComm() {
    for (int p = 0; p < kTpMaxRanks; ++p)
      if (peer[p]) cudaIpcCloseMemHandle(peer[p]);
    if (block) cudaFree(block);
    if (epoch) cudaFree(epoch);
  }
};

static int tp_comm_create(int rank, int n, int max_rows, int max_hidden, TpComm** out) {
  if (n < 1 || n > kTpMaxRanks || rank < 0 || rank >= n || max_rows < 1 || max_hidden < 8 || max_hidden % 8)
    return set_error(LMX_ERR_INVALID, "tp_comm: bad arguments (size <= %d, hidden %% 8 == 0)", kTpMaxRanks);
  auto c = std::make_unique<TpComm>();
  c->n = n;
  c->rank = rank;
  c->max_rows = max_rows;
  c->max_hidden = max_hidden;
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  c->t.n = n;
  c->t.rank = rank;
  c->t.slot_bytes = up((size_t)max_rows * max_hidden * sizeof(bf16_t));
  c->t.pairs_off = 2 * c->t.slot_bytes;
  c->t.flags_off = c->t.pairs_off + up((size_t)max_rows * 8);
  const size_t bytes = c->t.flags_off + up((size_t)kTpSlots * kTpMaxRanks * 4);
  c->block_bytes = bytes;
  int rc = cuda_check(cudaMalloc(&c->block, bytes), "tp_comm: block");
  if (!rc) rc = cuda_check(cudaMemset(c->block, 0, bytes), "tp_comm: zero");
  if (!rc) rc = cuda_check(cudaMalloc(&c->epoch, (size_t)kTpSlots * 4), "tp_comm: epoch");
  if (!rc) rc = cuda_check(cudaMemset(c->epoch, 0, (size_t)kTpSlots * 4), "tp_comm: zero");
  if (!rc) rc = cuda_check(cudaDeviceSynchronize(), "tp_comm: init");
  if (rc) return rc;
  c->t.base[rank] = (uint8_t*)c->block;
  c->t.epoch = c->epoch;
  c->opened = n == 1;
  *out = c.release();
  return LMX_OK;
}

// handles: n cudaIpcMemHandle_t blobs in rank order (this rank's is skipped).
static int tp_comm_open(TpComm& c, const void* handles) {
  if (c.opened) return set_error(LMX_ERR_INVALID, "tp_comm: already open");
  for (int p = 0; p < c.n; ++p) {
    if (p == c.rank || c.attached[p]) continue;
    cudaIpcMemHandle_t hd;
    std::memcpy(&hd, (const uint8_t*)handles + (size_t)p * sizeof(cudaIpcMemHandle_t), sizeof(hd));
    int rc = cuda_check(cudaIpcOpenMemHandle(&c.peer[p], hd, cudaIpcMemLazyEnablePeerAccess),
                        "tp_comm: open peer handle");
    if (rc) return rc;
    c.t.base[p] = (uint8_t*)c.peer[p];
  }
  c.opened = true;
  return LMX_OK;
}

// Attach peer `p`'s block by a device pointer this process can already
// address (a mapping the caller made itself).  The comm is open once every
// peer is attached or opened.
static int tp_comm_attach(TpComm& c, int p, void* block) {
  if (c.opened) return set_error(LMX_ERR_INVALID, "tp_comm: already open");
  if (p < 0 || p >= c.n || p == c.rank || !block || ((uintptr_t)block & 255))
    return set_error(LMX_ERR_INVALID, "tp_comm_attach: bad peer %d or unaligned block", p);
  c.t.base[p] = (uint8_t*)block;
  c.attached[p] = true;
  bool all = true;
  for (int q = 0; q < c.n; ++q) all = all && (q == c.rank || c.attached[q] || c.peer[q]);
  c.opened = all;
  return LMX_OK;
}

static bf16_t* tp_slot(const TpComm& c, int sel) {
  return (bf16_t*)((uint8_t*)c.block + (size_t)sel * c.t.slot_bytes);
}

static int launch_tp_allreduce_norm(const TpComm& c, int sel, int R, int H, bf16_t* h, const bf16_t* w, float eps,
                                    bf16_t* xn, cudaStream_t st) {
  if (R > c.max_rows || H > c.max_hidden) return set_error(LMX_ERR_INVALID, "tp all-reduce: %dx%d exceeds comm", R, H);
  static bool attr_set[64] = {};
  int d = 0;
  cudaGetDevice(&d);
  const size_t smem = (size_t)H * sizeof(bf16_t);
  if (!attr_set[d & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(tp_allreduce_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             64 * 1024),
                        "tp all-reduce: smem");
    if (rc) return rc;
    attr_set[d & 63] = true;
  }
  if (smem > 64 * 1024) return set_error(LMX_ERR_UNSUPPORTED, "tp all-reduce: hidden %d too large", H);
  const int grid = R < kTpArCtas ? R : kTpArCtas;
  return cuda_check(lmx_launch(tp_allreduce_norm_kernel, dim3(grid), dim3(256), smem, st, true, c.t, sel, R, H, h, w,
                               eps, xn, device_error_word()),
                    "tp all-reduce: launch");
}

// Vocab-parallel argmax: rows of this rank's logits slice [rows][ld] (V local
// columns starting at global index base) -> out[rows] global argmax.
static int launch_tp_argmax(const TpComm& c, const bf16_t* logits, int rows, int V, int ld, int base, int32_t* out,
                            cudaStream_t st) {
  if (rows > c.max_rows || rows > 1024) return set_error(LMX_ERR_INVALID, "tp argmax: %d rows", rows);
  uint2* pairs = (uint2*)((uint8_t*)c.block + c.t.pairs_off);
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
  int rc = cuda_check(lmx_counted(cudaLaunchKernelEx(&cfg, tp_argmax_local_kernel, logits, V, ld, base, pairs)),
                      "tp argmax: launch");
  if (rc) return rc;
  const int threads = rows < 32 ? 32 : (rows + 31) / 32 * 32;
  return cuda_check(lmx_launch(tp_argmax_exchange_kernel, dim3(1), dim3(threads), 0, st, true, c.t, rows, out,
                               device_error_word()),
                    "tp argmax exchange: launch");
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
struct QWeight {
  uint32_t* w = nullptr;
  bf16_t* s = nullptr;
  bf16_t* b = nullptr;
  int N = 0, K = 0;
  int bits = 4;  // this weight's quantization (a checkpoint may override it per layer)
  QMat mat() const {
    QMat m;
    m.w = w;
    m.s = s;
    m.b = b;
    m.rows = N;
    return m;
  }
};

struct Layer {
  QWeight w[7];  // q k v o gate up down
  bf16_t *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
};

struct Model {
  lmx_model_config c;
  int n_layers = 0;  // layers this (possibly view) model runs
  std::vector<Layer> L;
  QWeight embed, lm_head;
  bf16_t* final_norm = nullptr;
  float *cos_t = nullptr, *sin_t = nullptr;
  int max_pos = 16384;
  std::shared_ptr<Arena> arena;  // shared by views
  // tensor parallelism: this rank's share of the heads, FFN columns and
  // vocabulary rows (the whole model when tp == 1); comm is not owned
  int tp = 1, tp_rank = 0;
  TpComm* comm = nullptr;
  int hq = 0, hk = 0, il = 0, vl = 0;
  QWeight head_tp;  // vocab rows [tp_rank*vl, +vl) of the lm_head (tp > 1)
  bool uniform_bits = true;  // every weight at c.bits (the fused decode kernel's precondition)
  const QWeight& head() const { return tp > 1 ? head_tp : (c.tied ? embed : lm_head); }
};

// Rows [row0, row0+N) x columns [col0, col0+K) of tensor tid, a [*, Kfull]
// matrix (Kfull 0: the block is the whole width K).
static int gen_qweight(Arena& ar, QWeight& q, uint64_t seed, uint32_t tid, int N, int K, int bits,
                       cudaStream_t st, int64_t row0 = 0, int64_t col0 = 0, int64_t Kfull = 0) {
  q.N = N;
  q.K = K;
  q.bits = bits;
  int rc = ar.alloc(&q.w, (size_t)N * K * bits / 32, false);
  if (!rc) rc = ar.alloc(&q.s, (size_t)N * (K / 64), false);
  if (!rc) rc = ar.alloc(&q.b, (size_t)N * (K / 64), false);
  if (rc) return rc;
  const float C = (float)((double)0.02f * std::sqrt(3.0) / 4194304.0);
  const int64_t groups = (int64_t)N * (K / 64);
  gen_qweight_kernel<<<(unsigned)((groups + 127) / 128), 128, 0, st>>>(seed, tid, N, K, bits, C, row0, col0,
                                                                        Kfull ? Kfull : K, q.w, q.s, q.b);
  return cuda_check(cudaGetLastError(), "gen_qweight");
}

static int fill_ones(Arena& ar, bf16_t** p, int n, cudaStream_t st) {
  int rc = ar.alloc(p, n, false);
  if (rc) return rc;
  fill_bf16_kernel<<<(n + 255) / 256, 256, 0, st>>>(*p, n, (bf16_t)0x3F80);
  return cuda_check(cudaGetLastError(), "fill");
}

// Where model_build takes its tensors from: the seeded generator below or
// a checkpoint (loader.cuh).  qweight fills rows [row0, row0+N) x columns
// [col0, col0+K) of the named [Nfull, Kfull] linear weight (tid: the seeded
// tensor id); norm fills n values of the named vector.
struct WeightSource {
  virtual ~WeightSource() = default;
  virtual int qweight(Arena& ar, QWeight& q, uint32_t tid, const std::string& name, int N, int K, int64_t row0,
                      int64_t col0, int64_t Nfull, int64_t Kfull, cudaStream_t st) = 0;
  virtual int norm(Arena& ar, bf16_t** p, const std::string& name, int n, cudaStream_t st) = 0;
};

// Synthetic weights: N(0, 0.02) quantized at the config's bits; norms ones.
struct SeededSource : WeightSource {
  uint64_t seed;
  int bits;
  SeededSource(uint64_t s, int b) : seed(s), bits(b) {}
  int qweight(Arena& ar, QWeight& q, uint32_t tid, const std::string&, int N, int K, int64_t row0, int64_t col0,
              int64_t, int64_t Kfull, cudaStream_t st) override {
    return gen_qweight(ar, q, seed, tid, N, K, bits, st, row0, col0, Kfull);
  }
  int norm(Arena& ar, bf16_t** p, const std::string&, int n, cudaStream_t st) override {
    return fill_ones(ar, p, n, st);
  }
};

// comm == nullptr (or a size-1 comm): the whole model.  Otherwise this
// rank's tensor-parallel shard (Megatron split, tp.cuh): q/k/v by heads,
// gate/up by FFN rows, o/down by the matching input columns, the lm_head by
// vocabulary rows (a view into the packed embedding when tied); embedding
// table and norms are replicated.  Every shard holds exactly the values of
// its block of the unsharded weights.  Tensor names are the MLX checkpoint's
// (Qwen3Model / LlamaModel::weight_map, src/llm/models/qwen3.cpp:100-160,
// :236-241).
static int model_build(const lmx_model_config& c, WeightSource& src, TpComm* comm, Model** out) {
  if (c.group_size != 64 || (c.bits != 4 && c.bits != 8) || c.head_dim != kHeadDim ||
      c.hidden % 512 || c.heads % c.kv_heads || c.layers < 1 || c.vocab < 1)
    return set_error(LMX_ERR_UNSUPPORTED, "model config not supported (head_dim 128, hidden %% 512 == 0, group 64, 4/8-bit)");
  const int tp = comm ? comm->n : 1, r = comm ? comm->rank : 0;
  if (tp > 1) {
    if (!comm->opened) return set_error(LMX_ERR_INVALID, "model_create: tp comm not opened");
    if (c.heads % tp || c.kv_heads % tp || c.inter % (64 * tp) || c.vocab % tp || c.hidden > comm->max_hidden)
      return set_error(LMX_ERR_UNSUPPORTED,
                       "model_create: tp=%d needs heads, kv_heads, vocab %% tp == 0, inter %% (64 tp) == 0, "
                       "hidden <= comm max_hidden", tp);
  }
  auto m = std::make_unique<Model>();
  m->c = c;
  m->n_layers = c.layers;
  m->tp = tp;
  m->tp_rank = r;
  m->comm = tp > 1 ? comm : nullptr;
  m->hq = c.heads / tp;
  m->hk = c.kv_heads / tp;
  m->il = c.inter / tp;
  m->vl = c.vocab / tp;
  m->arena = std::make_shared<Arena>();
  Arena& ar = *m->arena;
  const int H = c.hidden, D = c.head_dim, I = c.inter, NQ = c.heads * D, NK = c.kv_heads * D;
  const int nq = m->hq * D, nk = m->hk * D, il = m->il;
  cudaStream_t st = 0;
  static const char* const kProj[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                       "mlp.gate_proj",    "mlp.up_proj",      "mlp.down_proj"};
  m->L.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const std::string pre = "model.layers." + std::to_string(l) + ".";
    // {rows, cols, row0, col0, full rows, full width}
    const int64_t shp[7][6] = {{nq, H, (int64_t)r * nq, 0, NQ, H},  {nk, H, (int64_t)r * nk, 0, NK, H},
                               {nk, H, (int64_t)r * nk, 0, NK, H},  {H, nq, 0, (int64_t)r * nq, H, NQ},
                               {il, H, (int64_t)r * il, 0, I, H},   {il, H, (int64_t)r * il, 0, I, H},
                               {H, il, 0, (int64_t)r * il, H, I}};
    for (int k = 0; k < 7; ++k) {
      int rc = src.qweight(ar, m->L[l].w[k], (uint32_t)((l + 1) * 16 + k), pre + kProj[k], (int)shp[k][0],
                           (int)shp[k][1], shp[k][2], shp[k][3], shp[k][4], shp[k][5], st);
      if (rc) return rc;
    }
    const Layer& Ly = m->L[l];
    if (Ly.w[0].bits != Ly.w[1].bits || Ly.w[0].bits != Ly.w[2].bits || Ly.w[4].bits != Ly.w[5].bits)
      return set_error(LMX_ERR_UNSUPPORTED,
                       "layer %d: q/k/v (and gate/up) run as one fused GEMM and must share their bits", l);
    int rc = src.norm(ar, &m->L[l].in_norm, pre + "input_layernorm.weight", H, st);
    if (!rc) rc = src.norm(ar, &m->L[l].post_norm, pre + "post_attention_layernorm.weight", H, st);
    if (!rc && c.qk_norm) rc = src.norm(ar, &m->L[l].q_norm, pre + "self_attn.q_norm.weight", D, st);
    if (!rc && c.qk_norm) rc = src.norm(ar, &m->L[l].k_norm, pre + "self_attn.k_norm.weight", D, st);
    if (rc) return rc;
  }
  int rc = src.qweight(ar, m->embed, 1, "model.embed_tokens", c.vocab, H, 0, 0, c.vocab, H, st);
  if (!rc && !c.tied) {
    if (tp == 1) rc = src.qweight(ar, m->lm_head, 2, "lm_head", c.vocab, H, 0, 0, c.vocab, H, st);
    else rc = src.qweight(ar, m->head_tp, 2, "lm_head", m->vl, H, (int64_t)r * m->vl, 0, c.vocab, H, st);
  } else if (!rc && tp > 1) {  // vocab rows of the tied table
    QWeight& v = m->head_tp;
    v.N = m->vl;
    v.K = H;
    v.bits = m->embed.bits;
    v.w = m->embed.w + (size_t)r * m->vl * (H * v.bits / 32);
    v.s = m->embed.s + (size_t)r * m->vl * (H / 64);
    v.b = m->embed.b + (size_t)r * m->vl * (H / 64);
  }
  if (!rc) rc = src.norm(ar, &m->final_norm, "model.norm.weight", H, st);
  if (rc) return rc;
  m->uniform_bits = true;
  for (const Layer& Ly : m->L)
    for (const QWeight& q : Ly.w) m->uniform_bits = m->uniform_bits && q.bits == c.bits;
  m->uniform_bits = m->uniform_bits && m->embed.bits == c.bits && m->head().bits == c.bits;
  // RoPE table: period_i = base^(2i/D) (with the Llama-3 frequency scaling of
  // LlamaDynamicNTKScalingRoPE::compute_freqs, src/llm/models/llama.cpp:122-183,
  // when rope_factor > 1), theta = pos / period (double), fp32 cos/sin
  std::vector<double> period(D / 2);
  for (int i = 0; i < D / 2; ++i) {
    double pd = std::pow((double)c.rope_theta, 2.0 * (double)i / (double)D);
    if (c.rope_factor > 1.0f) {
      const double wl = 2.0 * M_PI * pd;
      const double low_wl = (double)c.rope_orig_max_pos / (double)c.rope_low_freq;
      const double high_wl = (double)c.rope_orig_max_pos / (double)c.rope_high_freq;
      if (wl > low_wl) {
        pd = pd * (double)c.rope_factor;
      } else if (wl > high_wl) {
        const double s = ((double)c.rope_orig_max_pos / wl - (double)c.rope_low_freq) /
                         ((double)c.rope_high_freq - (double)c.rope_low_freq);
        pd = pd / ((1.0 - s) / (double)c.rope_factor + s);
      }
    }
    period[i] = pd;
  }
  std::vector<float> ct((size_t)m->max_pos * D / 2), stt(ct.size());
  for (int p = 0; p < m->max_pos; ++p)
    for (int i = 0; i < D / 2; ++i) {
      const double th = (double)p / period[i];
      ct[(size_t)p * D / 2 + i] = (float)std::cos(th);
      stt[(size_t)p * D / 2 + i] = (float)std::sin(th);
    }
  rc = ar.alloc(&m->cos_t, ct.size(), false);
  if (!rc) rc = ar.alloc(&m->sin_t, stt.size(), false);
  if (rc) return rc;
  rc = cuda_check(cudaMemcpy(m->cos_t, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice), "rope table");
  if (!rc) rc = cuda_check(cudaMemcpy(m->sin_t, stt.data(), stt.size() * 4, cudaMemcpyHostToDevice), "rope table");
  if (!rc) rc = cuda_check(cudaDeviceSynchronize(), "model init");
  if (rc) return rc;
  *out = m.release();
  return LMX_OK;
}

static int model_create(const lmx_model_config& c, uint64_t seed, TpComm* comm, Model** out) {
  SeededSource src(seed, c.bits);
  return model_build(c, src, comm, out);
}

// ---------------------------------------------------------------------------
// KV cache (KVCacheSimple / QuantizedKVCache, src/common/kv_cache.cpp):
// preallocated to `capacity` rows; lengths live on the device.
// ---------------------------------------------------------------------------
struct Cache {
  int n_layers = 0, B = 0, cap = 0, bits = 16, Hk = 0;
  int hk0 = 0, Hk_total = 0;  // first KV head of this shard, KV heads of the whole model
  std::vector<KvDesc> kv;
  int* len = nullptr;
  DecLayer* dec = nullptr;  // per-layer weights + this cache, for the fused decode (device)
  Arena ar;
};

// Synthetic context (fill_kv_kernel): rows [0, n) of every layer's K and V,
// tensor ids tid_base + 2*layer + (0 K, 1 V), N(0,1); every length set to n.
static int cache_fill_synthetic(Cache& c, int n, uint64_t seed, uint32_t tid_base, cudaStream_t st) {
  if (n < 0 || n > c.cap) return set_error(LMX_ERR_INVALID, "fill_synthetic: %d rows > capacity %d", n, c.cap);
  const float C = (float)(std::sqrt(3.0) / 4194304.0);
  const int64_t threads = (int64_t)c.B * c.Hk * n * (kHeadDim / 64);
  for (int l = 0; l < c.n_layers && threads > 0; ++l)
    for (int v = 0; v < 2; ++v) {
      fill_kv_kernel<<<(unsigned)((threads + 127) / 128), 128, 0, st>>>(seed, tid_base + 2u * l + v, c.kv[l], v, n,
                                                                       c.hk0, c.Hk_total, C);
      int rc = cuda_check(cudaGetLastError(), "fill_kv");
      if (rc) return rc;
    }
  std::vector<int> lens(c.B, n);
  int rc = cuda_check(cudaMemcpyAsync(c.len, lens.data(), (size_t)c.B * 4, cudaMemcpyHostToDevice, st), "len");
  if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "fill_synthetic");
  return rc;
}

static int cache_create(const Model& m, int n_layers, int B, int cap, int bits, Cache** out) {
  if (bits != 16 && bits != 4 && bits != 8) return set_error(LMX_ERR_UNSUPPORTED, "kv_bits %d", bits);
  if (n_layers < 1 || n_layers > m.n_layers || B < 1 || cap < 1 || cap > m.max_pos)
    return set_error(LMX_ERR_INVALID, "cache: bad arguments");
  auto c = std::make_unique<Cache>();
  c->n_layers = n_layers;
  c->B = B;
  // rows are allocated in whole 128-key splits: the fused decode stages a
  // split's rows with bulk copies that never cross into the next sequence
  cap = (cap + kSplit - 1) / kSplit * kSplit;
  c->cap = cap;
  c->bits = bits;
  c->Hk = m.hk;
  c->hk0 = m.tp_rank * m.hk;
  c->Hk_total = m.c.kv_heads;
  int rc = c->ar.alloc(&c->len, B);
  if (rc) return rc;
  const size_t rows = (size_t)B * c->Hk * cap;
  c->kv.resize(n_layers);
  for (int l = 0; l < n_layers; ++l) {
    KvDesc& d = c->kv[l];
    std::memset(&d, 0, sizeof(d));
    d.B = B;
    d.Hk = c->Hk;
    d.cap = cap;
    d.bits = bits;
    d.len = c->len;
    if (bits == 16) {
      rc = c->ar.alloc(&d.k, rows * kHeadDim);
      if (!rc) rc = c->ar.alloc(&d.v, rows * kHeadDim);
    } else {
      rc = c->ar.alloc(&d.kq, rows * kHeadDim * bits / 32);
      if (!rc) rc = c->ar.alloc(&d.vq, rows * kHeadDim * bits / 32);
      if (!rc) rc = c->ar.alloc(&d.ks, rows * 2);
      if (!rc) rc = c->ar.alloc(&d.kb, rows * 2);
      if (!rc) rc = c->ar.alloc(&d.vs, rows * 2);
      if (!rc) rc = c->ar.alloc(&d.vb, rows * 2);
    }
    if (rc) return rc;
  }
  // layer descriptors of the fused decode: the model's weights with this cache
  // (none for a geometry-only model)
  if ((int)m.L.size() < n_layers) {
    *out = c.release();
    return LMX_OK;
  }
  std::vector<DecLayer> dl(n_layers);
  for (int l = 0; l < n_layers; ++l) {
    DecLayer& d = dl[l];
    std::memset(&d, 0, sizeof(d));
    for (int k = 0; k < 7; ++k) d.m[k] = m.L[l].w[k].mat();
    d.in_norm = m.L[l].in_norm;
    d.post_norm = m.L[l].post_norm;
    d.q_norm = m.c.qk_norm ? m.L[l].q_norm : nullptr;
    d.k_norm = m.c.qk_norm ? m.L[l].k_norm : nullptr;
    d.kv = c->kv[l];
  }
  rc = c->ar.alloc(&c->dec, (size_t)n_layers, false);
  if (!rc) rc = cuda_check(cudaMemcpy(c->dec, dl.data(), dl.size() * sizeof(DecLayer), cudaMemcpyHostToDevice),
                           "cache: decode layers");
  if (rc) return rc;
  *out = c.release();
  return LMX_OK;
}

}  // namespace lmx

namespace lmx {

// ---------------------------------------------------------------------------
// activation workspace (sized at setup for the largest forward)
// ---------------------------------------------------------------------------
static constexpr int kPrefillChunk = 32;

struct Workspace {
  int Rmax = 0, tiles = 0, splits = 0, B = 0, Hk = 0;
  size_t part_floats = 0, n_counters = 0;
  bf16_t *h = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *o = nullptr, *act = nullptr,
         *logits = nullptr;
  float* part = nullptr;
  unsigned* counters = nullptr;
  // fused decode: split-K partial tiles, per-tile counters, grid-barrier counters
  float* dgpart = nullptr;
  unsigned* dgcnt = nullptr;
  unsigned* dbar = nullptr;
  size_t dgpart_floats = 0;
  int dgcnt_n = 0;
  Arena ar;
};

// Process-wide switch of the fused small-batch decode (tensor-core mode only).
// Off by default: measured on the B200 it is slower than the per-op kernels
// (a Qwen3-0.6B draft token at B = 8 over a 900-row 4-bit cache: 4.3 ms fused
// against 2.3 ms; each phase is bound by its ~2-4 us of per-item latency and
// ~3 us grid barriers, not by HBM).
static int g_fused_decode = 0;

// Reserve the fused decode's scratch in ws for model m at up to R rows.
static int dec_ws_reserve(Workspace& ws, const Model& m, int R) {
  if (R > kDecMaxRows) R = kDecMaxRows;
  DecPlan p;
  if (!dec_plan(m.c.hidden, m.hq, m.hk, m.il, R, device_sms(), p)) return LMX_OK;  // never fused
  int rc = LMX_OK;
  if (p.gpart_floats > ws.dgpart_floats) {
    rc = ws.ar.alloc(&ws.dgpart, p.gpart_floats, false);
    if (!rc) ws.dgpart_floats = p.gpart_floats;
  }
  if (!rc && p.max_tiles > ws.dgcnt_n) {
    rc = ws.ar.alloc(&ws.dgcnt, (size_t)p.max_tiles);
    if (!rc) ws.dgcnt_n = p.max_tiles;
  }
  if (!rc && !ws.dbar) rc = ws.ar.alloc(&ws.dbar, 2);
  return rc;
}

// Sized by m's per-rank shapes (hq, hk, il, vl; hidden from m.c).
static int workspace_create(const Model& m, int B, int Tmax, int cap, int logit_rows, Workspace& ws) {
  const lmx_model_config& c = m.c;
  const int R = B * Tmax, NQ = m.hq * kHeadDim, NK = m.hk * kHeadDim;
  const int G = m.hq / m.hk;
  ws.Rmax = R;
  ws.B = B;
  ws.Hk = m.hk;
  ws.tiles = (G * Tmax + kRowTile - 1) / kRowTile;
  ws.splits = (cap + kSplit - 1) / kSplit;
  int rc = ws.ar.alloc(&ws.h, (size_t)R * c.hidden);
  if (!rc) rc = ws.ar.alloc(&ws.xn, (size_t)R * (c.hidden > m.il ? c.hidden : m.il));
  if (!rc) rc = ws.ar.alloc(&ws.qkv, (size_t)R * (NQ + 2 * NK));
  if (!rc) rc = ws.ar.alloc(&ws.q, (size_t)R * NQ);
  if (!rc) rc = ws.ar.alloc(&ws.o, (size_t)R * NQ);
  if (!rc) rc = ws.ar.alloc(&ws.act, (size_t)R * m.il);
  if (!rc) rc = ws.ar.alloc(&ws.logits, (size_t)logit_rows * m.vl);
  cap = (cap + kSplit - 1) / kSplit * kSplit;  // as the caches round it
  sdpa_scratch_need(B, Tmax, G, m.hk, cap, ws.part_floats, ws.n_counters);
  if (!rc) rc = ws.ar.alloc(&ws.part, ws.part_floats, false);
  if (!rc) rc = ws.ar.alloc(&ws.counters, ws.n_counters);
  return rc;
}

// The fused decode forward applies: tensor-core mode, no tensor parallelism,
// R <= 16 rows, shapes the plan supports, scratch reserved, one CTA per SM fits.
static bool dec_applies(const Model& m, const Cache& c, int n_layers, int B, int T, const Workspace& ws,
                        DecPlan& p) {
  const int R = B * T, G = m.hq / m.hk;
  if (!g_fused_decode || m.tp > 1 || qmm_mma_min_m() <= 0 || R < 1 || R > kDecMaxRows || G * T > kDecAttnRows)
    return false;
  if ((m.c.bits != 4 && m.c.bits != 8) || !m.uniform_bits || !c.dec || c.cap % kSplit || n_layers > c.n_layers)
    return false;
  if (!dec_plan(m.c.hidden, m.hq, m.hk, m.il, R, device_sms(), p)) return false;
  if (p.gpart_floats > ws.dgpart_floats || p.max_tiles > ws.dgcnt_n || !ws.dbar) return false;
  const size_t need = (size_t)B * m.hk * (c.cap / kSplit) * kRowTile * kPartStride;
  if (need > ws.part_floats || (size_t)B * m.hk > ws.n_counters) return false;
  return dec_occupancy_for(m.c.bits, R) >= 1;
}

// One forward of T tokens per sequence through layers [0, n_layers) of m,
// appending K/V at each sequence's device-side cache length (the caller
// advances the lengths).  Per layer: qkv GEMV (+fused RMSNorm) -> q/k norm,
// RoPE, KV append -> SDPA -> o_proj GEMV (+residual) -> gate|up GEMV
// (+RMSNorm, SwiGLU) -> down GEMV (+residual); then the final norm and the
// lm_head for every row or only each sequence's last row.
// Tensor-parallel shard (m.tp > 1): o_proj and down write this rank's
// partial into the comm's slot and tp_allreduce_norm_kernel adds the sum to
// the residual and applies the next RMSNorm (post-attention, the next
// layer's input norm, or the final norm); the lm_head produces this rank's
// vocabulary slice [rows][vl].
static int forward(const Model& m, Cache& c, int n_layers, const int32_t* tok, int tok_ld, int tok_off,
                   int B, int T, Workspace& ws, bf16_t* logits, bool last_only, cudaStream_t st,
                   int logits_ld = 0) {
  const lmx_model_config& cf = m.c;
  const int H = cf.hidden, I = m.il, Hq = m.hq, Hk = m.hk;
  const int NQ = Hq * kHeadDim, NK = Hk * kHeadDim, G = Hq / Hk, R = B * T;
  const bool tp = m.tp > 1;
  if (R > ws.Rmax || B != c.B || n_layers > c.n_layers || n_layers > m.n_layers || c.Hk != Hk)
    return set_error(LMX_ERR_INVALID, "forward: shape exceeds workspace");
  const int tiles = (G * T + kRowTile - 1) / kRowTile, splits = (c.cap + kSplit - 1) / kSplit;
  if (tiles > ws.tiles || splits > ws.splits || B > ws.B || Hk > ws.Hk)
    return set_error(LMX_ERR_INVALID, "forward: attention scratch too small");
  if (tp && (R > m.comm->max_rows || H > m.comm->max_hidden))
    return set_error(LMX_ERR_INVALID, "forward: %d rows exceed the tp comm", R);
  // the input / post-attention RMSNorm fused into the GEMV prologue (both
  // GEMV paths; the tcgen05 path takes normalised rows through TMA)
  const bool fuse = !tp && R <= kQmmMaxNormRows && !qmm_uses_mma(R);
  int rc = cuda_check(lmx_launch(embed_kernel, dim3(R), dim3(256), 0, st, true, tok, T, tok_ld, tok_off,
                                 (const uint32_t*)m.embed.w, (const bf16_t*)m.embed.s,
                                 (const bf16_t*)m.embed.b, H, m.embed.bits, ws.h, R),
                      "embed");
  if (rc) return rc;
  const float scale = (float)(1.0 / std::sqrt((double)kHeadDim));
  int dummy_sel = 0;
  int& sel = tp ? m.comm->sel : dummy_sel;  // tp partial slot, alternating per exchange on the comm
  DecPlan dp;
  if (dec_applies(m, c, n_layers, B, T, ws, dp)) {
    // the whole layer stack in one persistent launch (decode.cuh)
    DecArgs da;
    da.L = c.dec;
    da.nl = n_layers;
    da.B = B;
    da.T = T;
    da.R = R;
    da.H = H;
    da.Hq = Hq;
    da.Hk = Hk;
    da.I = I;
    for (int ph = 0; ph < kDecPhases; ++ph) da.ks[ph] = dp.ks[ph];
    da.nsplit = c.cap / kSplit;
    da.eps = cf.eps;
    da.scale = scale;
    da.cos_t = m.cos_t;
    da.sin_t = m.sin_t;
    da.max_pos = m.max_pos;
    da.h = ws.h;
    da.qkv = ws.qkv;
    da.o = ws.o;
    da.act = ws.act;
    da.gpart = ws.dgpart;
    da.gcnt = ws.dgcnt;
    da.apart = ws.part;
    da.acnt = ws.counters;
    da.bar = ws.dbar;
    da.err = device_error_word();
    rc = dec_launch(da, cf.bits, st);
    n_layers = 0;  // the per-op loop below has nothing left to do
  }
  for (int l = 0; l < n_layers && !rc; ++l) {
    const Layer& L = m.L[l];
    QmmCall qc;
    if (fuse) {
      qc.x = ws.h;
      qc.norm_w = L.in_norm;
    } else {
      // tp: layers > 0 get xn from the previous layer's all-reduce
      if (!tp || l == 0) rc = launch_rms_norm(ws.h, L.in_norm, ws.xn, R, H, cf.eps, st);
      qc.x = ws.xn;
    }
    qc.eps = cf.eps;
    qc.mat[0] = L.w[0].mat();
    qc.mat[1] = L.w[1].mat();
    qc.mat[2] = L.w[2].mat();
    qc.nmat = 3;
    qc.N = NQ + 2 * NK;
    qc.y = ws.qkv;
    qc.ldy = qc.N;
    qc.M = R;
    qc.K = H;
    qc.bits = L.w[0].bits;
    if (!rc) rc = launch_qmm(qc, st);

    PrepArgs pa;
    pa.qkv = ws.qkv;
    pa.ldq = NQ + 2 * NK;
    pa.R = R;
    pa.T = T;
    pa.Hq = Hq;
    pa.Hk = Hk;
    pa.qn = cf.qk_norm ? L.q_norm : nullptr;
    pa.kn = cf.qk_norm ? L.k_norm : nullptr;
    pa.eps = cf.eps;
    pa.cos_t = m.cos_t;
    pa.sin_t = m.sin_t;
    pa.max_pos = m.max_pos;
    pa.q_out = ws.q;
    pa.kv = c.kv[l];
    pa.err = device_error_word();
    if (!rc) rc = launch_attn_prep(pa, st);

    SdpaArgs sa;
    sa.q = ws.q;
    sa.kv = c.kv[l];
    sa.T = T;
    sa.Hq = Hq;
    sa.scale = scale;
    sa.nsplit = splits;
    sa.tiles = tiles;
    sa.part = ws.part;
    sa.counters = ws.counters;
    sa.part_floats = ws.part_floats;
    sa.n_counters = ws.n_counters;
    sa.err = device_error_word();
    sa.out = ws.o;
    if (!rc) rc = launch_sdpa(sa, B, st);

    QmmCall oc;
    oc.x = ws.o;
    oc.mat[0] = L.w[3].mat();
    oc.N = H;
    oc.ldy = H;
    oc.M = R;
    oc.K = NQ;
    oc.bits = L.w[3].bits;
    if (tp) {
      oc.y = tp_slot(*m.comm, sel);
      oc.mode = kPlain;
      if (!rc) rc = launch_qmm(oc, st);
      if (!rc) rc = launch_tp_allreduce_norm(*m.comm, sel, R, H, ws.h, L.post_norm, cf.eps, ws.xn, st);
      sel ^= 1;
    } else {
      oc.y = ws.h;
      oc.res = ws.h;
      oc.mode = kResid;
      if (!rc) rc = launch_qmm(oc, st);
    }

    QmmCall gc;
    if (fuse) {
      gc.x = ws.h;
      gc.norm_w = L.post_norm;
    } else {
      if (!tp && !rc) rc = launch_rms_norm(ws.h, L.post_norm, ws.xn, R, H, cf.eps, st);
      gc.x = ws.xn;
    }
    gc.eps = cf.eps;
    gc.mat[0] = L.w[4].mat();
    gc.mat[1] = L.w[5].mat();
    gc.nmat = 2;
    gc.N = I;
    gc.y = ws.act;
    gc.ldy = I;
    gc.M = R;
    gc.K = H;
    gc.bits = L.w[4].bits;
    gc.mode = kSwiglu;
    if (!rc) rc = launch_qmm(gc, st);

    QmmCall dc;
    dc.x = ws.act;
    dc.mat[0] = L.w[6].mat();
    dc.N = H;
    dc.ldy = H;
    dc.M = R;
    dc.K = I;
    dc.bits = L.w[6].bits;
    if (tp) {
      dc.y = tp_slot(*m.comm, sel);
      dc.mode = kPlain;
      const bf16_t* next_norm = l + 1 < n_layers ? m.L[l + 1].in_norm : m.final_norm;
      if (!rc) rc = launch_qmm(dc, st);
      if (!rc) rc = launch_tp_allreduce_norm(*m.comm, sel, R, H, ws.h, next_norm, cf.eps, ws.xn, st);
      sel ^= 1;
    } else {
      dc.y = ws.h;
      dc.res = ws.h;
      dc.mode = kResid;
      if (!rc) rc = launch_qmm(dc, st);
    }
  }
  if (rc || !logits) return rc;
  QmmCall hc;
  const int M = last_only ? B : R;
  const bf16_t* src = ws.h;
  if (tp) {
    src = ws.xn;  // final-normed by the last all-reduce
  } else if (M > kQmmMaxNormRows || qmm_uses_mma(M)) {
    rc = launch_rms_norm(ws.h, m.final_norm, ws.xn, R, H, cf.eps, st);
    if (rc) return rc;
    src = ws.xn;
  } else {
    hc.norm_w = m.final_norm;
  }
  hc.x = last_only ? src + (size_t)(T - 1) * H : src;
  hc.ldx = last_only ? T * H : H;
  hc.eps = cf.eps;
  hc.mat[0] = m.head().mat();
  hc.N = m.vl;
  hc.y = logits;
  hc.ldy = logits_ld ? logits_ld : m.vl;
  hc.M = M;
  hc.K = H;
  hc.bits = m.head().bits;
  return launch_qmm(hc, st);
}

// Greedy token of each of `rows` logits rows (ld columns apart): the cluster
// argmax, or the vocab-parallel argmax across the ranks of a tp model.
static int model_argmax(const Model& m, const bf16_t* logits, int rows, int ld, int32_t* out, cudaStream_t st) {
  if (m.tp > 1) return launch_tp_argmax(*m.comm, logits, rows, m.vl, ld, m.tp_rank * m.vl, out, st);
  if (ld != m.vl) return set_error(LMX_ERR_INVALID, "argmax: ld %d != vocab %d", ld, m.vl);
  return launch_argmax(logits, rows, m.vl, out, st);
}

static int add_len(int* len, int B, int n, cudaStream_t st) {
  return cuda_check(lmx_launch(add_len_kernel, dim3((B + 127) / 128), dim3(128), 0, st, true, len, B, n),
                    "add_len");
}

// Forward a [B, T] token block in chunks (prefill), advancing the lengths.
static int forward_chunked(const Model& m, Cache& c, int n_layers, const int32_t* tok, int ld, int T, int B,
                           Workspace& ws, bf16_t* last_logits, cudaStream_t st) {
  int rc = LMX_OK;
  for (int t0 = 0; t0 < T && !rc; t0 += kPrefillChunk) {
    const int tn = T - t0 < kPrefillChunk ? T - t0 : kPrefillChunk;
    const bool last = t0 + tn >= T;
    rc = forward(m, c, n_layers, tok, ld, t0, B, tn, ws, last ? last_logits : nullptr, true, st);
    if (!rc) rc = add_len(c.len, B, tn, st);
  }
  return rc;
}

// ---------------------------------------------------------------------------
// speculative decoder
// ---------------------------------------------------------------------------
struct Spec {
  Model* tm = nullptr;
  Model* dm = nullptr;
  int dl = 0;
  lmx_spec_config cfg;
  std::unique_ptr<Cache> tc, dc;
  Workspace ws;
  SpecState s;
  int32_t *prompts = nullptr, *yprefill = nullptr;
  Arena ar;
  cudaStream_t st = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool prefilled = false;
  int64_t replays = 0;  // graph replays (steps enqueued) of the last decode
  // per-token iteration (lmx_spec_next): tokens read so far per sequence,
  // the device counts and stream mirrored after the last step
  std::vector<int> it_rp, it_em;
  std::vector<int32_t> it_buf;
  ~Spec() {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (st) cudaStreamDestroy(st);
  }
};

static StochParams stoch_params(const Spec& sp) {
  StochParams p;
  p.temperature = sp.cfg.temperature;
  p.top_p = sp.cfg.top_p;
  p.seed = sp.cfg.seed;
  p.seq_base = (uint32_t)sp.cfg.seq_base;
  return p;
}

static int spec_step(Spec& sp) {
  const int B = sp.cfg.batch, K = sp.cfg.K, V = sp.tm->c.vocab;
  cudaStream_t st = sp.st;
  const bool stoch = sp.cfg.temperature > 0.0f;
  int rc = LMX_OK;
  for (int i = 0; i < K && !rc; ++i) {
    const int32_t* tok = i == 0 ? sp.s.tok2 : sp.s.drafts;
    const int ld = i == 0 ? 2 : K, off = i == 0 ? 0 : i - 1, T = i == 0 ? 2 : 1;
    if (stoch) {
      rc = forward(*sp.dm, *sp.dc, sp.dl, tok, ld, off, B, T, sp.ws, sp.s.qlog + (size_t)i * V, true, st, K * V);
      if (!rc)
        rc = cuda_check(samp_launch(draft_sample_kernel, B, V, 1, st,
                                   (const bf16_t*)sp.s.qlog, V, sp.s, stoch_params(sp), i, T),
                        "draft_sample");
    } else {
      rc = forward(*sp.dm, *sp.dc, sp.dl, tok, ld, off, B, T, sp.ws, sp.ws.logits, true, st);
      if (sp.dm->tp > 1) {  // vocab-parallel argmax into the (free until the verify) pred rows
        if (!rc) rc = model_argmax(*sp.dm, sp.ws.logits, B, sp.dm->vl, sp.s.pred, st);
        if (!rc)
          rc = cuda_check(lmx_launch(draft_commit_kernel, dim3((B + 127) / 128), dim3(128), 0, st, true, sp.s,
                                     (const int32_t*)sp.s.pred, i, T),
                          "draft commit");
      } else if (!rc) {
        rc = launch_cluster_rows(draft_argmax_kernel, B, sp.ws.logits, V, sp.s, i, T, st);
      }
    }
  }
  if (!rc) rc = forward(*sp.tm, *sp.tc, sp.tm->n_layers, sp.s.vt, K + 1, 0, B, K + 1, sp.ws, sp.ws.logits, false, st);
  if (stoch) {
    if (!rc)
      rc = cuda_check(samp_launch(accept_stochastic_kernel, B, V, 2, st,
                                 (const bf16_t*)sp.ws.logits, V, sp.s, stoch_params(sp)),
                      "accept_stochastic");
  } else {
    if (!rc) rc = model_argmax(*sp.tm, sp.ws.logits, B * (K + 1), sp.tm->vl, sp.s.pred, st);
    if (!rc)
      rc = cuda_check(lmx_launch(accept_greedy_kernel, dim3((B + 127) / 128), dim3(128), 0, st, true, sp.s),
                      "accept");
  }
  return rc;
}

}  // namespace lmx

namespace lmx {

// The reference's KVCacheSimple allocation after prefilling n tokens: the
// prompt in chunks of 512 while more than 512 remain, then the rest
// (include/mlx-lm/llm/llm_model.h:18-60); first allocation max(chunk, 256)
// rows, then max(2 alloc, offset + chunk) when a chunk does not fit
// (src/common/kv_cache.cpp:34-110, include/mlx-lm/common/kv_cache.h:43).
static int kv_quirk_alloc(int n) {
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

static int spec_create(Model* tm, Model* dm, int dl, const lmx_spec_config& cfg, Spec** out) {
  if (cfg.batch < 1 || cfg.K < 0 || cfg.max_tokens < 1 || cfg.prompt_len < 2 || cfg.seq_base < 0)
    return set_error(LMX_ERR_INVALID, "spec: bad config");
  if (dm->c.vocab != tm->c.vocab) return set_error(LMX_ERR_INVALID, "spec: draft and target must share the vocabulary");
  // the draft runs replicated (tp 1) on every rank, or as this rank's shard
  // over the target's communicator
  if (dm->tp > 1 && (dm->tp != tm->tp || dm->comm != tm->comm))
    return set_error(LMX_ERR_UNSUPPORTED, "spec: a tensor-parallel draft shares the target's communicator");
  if ((tm->tp > 1 || dm->tp > 1) && cfg.temperature > 0.0f)
    return set_error(LMX_ERR_UNSUPPORTED, "spec: tensor-parallel models decode greedily (temperature 0)");
  auto sp = std::make_unique<Spec>();
  sp->tm = tm;
  sp->dm = dm;
  sp->dl = dl;
  sp->cfg = cfg;
  const int B = cfg.batch, K = cfg.K, P = cfg.prompt_len;
  if (cfg.context_len < 0) return set_error(LMX_ERR_INVALID, "spec: context_len < 0");
  const bool quirk = cfg.kv_quirk && cfg.kv_bits != 16;
  const int cap = (quirk ? kv_quirk_alloc(cfg.context_len + P) : cfg.context_len + P) + cfg.max_tokens + K + 8;
  Cache *tc = nullptr, *dc = nullptr;
  int rc = cache_create(*tm, tm->n_layers, B, cap, cfg.kv_bits, &tc);
  if (rc) return rc;
  sp->tc.reset(tc);
  // K = 0 is plain (non-speculative) decoding: the draft never runs
  rc = cache_create(*dm, K > 0 ? dl : 1, B, cap, cfg.kv_bits, &dc);
  if (rc) return rc;
  sp->dc.reset(dc);
  // one workspace serves both models: every dimension is the larger of the
  // two, the attention scratch is sized for the larger group (q heads per KV
  // head) and KV head count (its layout follows each call's own shape)
  Model shape;
  shape.c = tm->c;
  shape.c.hidden = std::max(tm->c.hidden, dm->c.hidden);
  shape.hk = std::max(tm->hk, dm->hk);
  shape.hq = std::max(tm->hq / tm->hk, dm->hq / dm->hk) * shape.hk;
  shape.il = std::max(tm->il, dm->il);
  shape.vl = std::max(tm->vl, dm->vl);
  const int Tmax = std::max(K + 1, kPrefillChunk);
  rc = workspace_create(shape, B, Tmax, cap, B * (K + 1), sp->ws);
  if (!rc) rc = dec_ws_reserve(sp->ws, *tm, kDecMaxRows);
  if (!rc) rc = dec_ws_reserve(sp->ws, *dm, kDecMaxRows);
  if (rc) return rc;
  SpecState& s = sp->s;
  s.B = B;
  s.K = K;
  s.max_tokens = cfg.max_tokens;
  rc = sp->ar.alloc(&s.tok2, (size_t)2 * B);
  if (!rc) rc = sp->ar.alloc(&s.drafts, (size_t)B * K);
  if (!rc) rc = sp->ar.alloc(&s.vt, (size_t)B * (K + 1));
  if (!rc) rc = sp->ar.alloc(&s.pred, (size_t)B * (K + 1));
  if (!rc) rc = sp->ar.alloc(&s.emitted, (size_t)B);
  if (!rc) rc = sp->ar.alloc(&s.accepted, (size_t)B);
  if (!rc) rc = sp->ar.alloc(&s.steps, (size_t)B);
  if (!rc) rc = sp->ar.alloc(&s.out, (size_t)B * cfg.max_tokens);
  s.qlog = nullptr;
  s.ustep = nullptr;
  if (!rc && cfg.temperature > 0.0f) {
    rc = sp->ar.alloc(&s.qlog, (size_t)B * K * tm->c.vocab);
    if (!rc) rc = sp->ar.alloc(&s.ustep, (size_t)B);
  }
  if (!rc) rc = sp->ar.alloc(&sp->prompts, (size_t)B * P);
  if (!rc) rc = sp->ar.alloc(&sp->yprefill, (size_t)B);
  if (rc) return rc;
  s.tlen = sp->tc->len;
  s.dlen = sp->dc->len;
  if (!rc) rc = cuda_check(cudaStreamCreateWithFlags(&sp->st, cudaStreamNonBlocking), "stream");
  if (rc) return rc;
  *out = sp.release();
  return LMX_OK;
}

static constexpr uint32_t kCtxTidTarget = 0x40000000u, kCtxTidDraft = 0x50000000u;

// Quantize rows [0, rows) of a bf16 cache layer into a 4/8-bit one (the
// append rule): one warp per (sequence, KV head, row, K or V).
__global__ void kv_quirk_convert_kernel(KvDesc src, KvDesc dst, int rows) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)src.B * src.Hk * rows * 2) return;
  const bool is_v = (w & 1) != 0;
  const int64_t r = w >> 1, bh = r / rows;
  const int j = (int)(r % rows);
  float x[8];
  if (lane < 16) unpack8(*reinterpret_cast<const uint4*>((is_v ? src.v : src.k) + ((size_t)bh * src.cap + j) * kHeadDim + 8 * lane), x);
  else
    for (int e = 0; e < 8; ++e) x[e] = 0.0f;
  uint4 deq;
  dec_append(dst, !is_v, (size_t)bh * dst.cap + j, lane, x, deq);
}

// Prefill for the KV pad quirk: the prompt into bf16 copies of both caches,
// then the reference allocation quantized into the real caches.
static int quirk_convert(Cache& src, Cache& dst, int rows, cudaStream_t st) {
  if (rows > dst.cap || rows > src.cap) return set_error(LMX_ERR_CAPACITY, "kv quirk: %d rows > capacity", rows);
  const int64_t threads = (int64_t)src.B * src.Hk * rows * 2 * 32;
  for (int l = 0; l < dst.n_layers; ++l) {
    kv_quirk_convert_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(src.kv[l], dst.kv[l], rows);
    int rc = cuda_check(cudaGetLastError(), "kv quirk convert");
    if (rc) return rc;
  }
  return LMX_OK;
}

// Prefill (TokenIterator::prepare, src/common/generate.cpp:508-549): the
// target runs the prompt and its argmax at the last position is d0 of the
// first step; the draft runs prompt[0, P-1) (its first step re-runs P-1).
static int spec_prefill(Spec& sp, const int32_t* prompts_host) {
  const int B = sp.cfg.batch, P = sp.cfg.prompt_len;
  cudaStream_t st = sp.st;
  int rc = cuda_check(cudaMemcpyAsync(sp.prompts, prompts_host, (size_t)B * P * 4, cudaMemcpyHostToDevice, st),
                      "prompts");
  const int ctx = sp.cfg.context_len;
  const bool quirk = sp.cfg.kv_quirk && sp.cfg.kv_bits != 16;
  const int tl = quirk ? kv_quirk_alloc(ctx + P) : ctx + P, dl = quirk ? kv_quirk_alloc(ctx + P - 1) : ctx + P - 1;
  // the KV pad quirk prefills into bf16 copies of the caches
  std::unique_ptr<Cache> tq, dq;
  if (!rc && quirk) {
    Cache *a = nullptr, *b = nullptr;
    rc = cache_create(*sp.tm, sp.tc->n_layers, B, sp.tc->cap, 16, &a);
    tq.reset(a);
    if (!rc) rc = cache_create(*sp.dm, sp.dc->n_layers, B, sp.dc->cap, 16, &b);
    dq.reset(b);
  }
  Cache& tpre = quirk ? *tq : *sp.tc;
  Cache& dpre = quirk ? *dq : *sp.dc;
  // the synthetic context (if any) precedes the prompt in both caches
  if (!rc) rc = cache_fill_synthetic(tpre, ctx, sp.cfg.context_seed, kCtxTidTarget, st);
  if (!rc) rc = cache_fill_synthetic(dpre, ctx, sp.cfg.context_seed, kCtxTidDraft, st);
  if (!rc) rc = forward_chunked(*sp.tm, tpre, sp.tm->n_layers, sp.prompts, P, P, B, sp.ws, sp.ws.logits, st);
  if (!rc && sp.cfg.temperature > 0.0f)
    rc = cuda_check(samp_launch(sample_rows_kernel, B, sp.tm->c.vocab, 1, st,
                               (const bf16_t*)sp.ws.logits, sp.tm->c.vocab, sp.tm->c.vocab, stoch_params(sp),
                               0u, 0u, 3u, sp.yprefill),
                    "prefill sample");
  else if (!rc)
    rc = model_argmax(*sp.tm, sp.ws.logits, B, sp.tm->vl, sp.yprefill, st);
  if (!rc && sp.cfg.K > 0) rc = forward_chunked(*sp.dm, dpre, sp.dl, sp.prompts, P, P - 1, B, sp.ws, nullptr, st);
  if (!rc && quirk) {
    rc = quirk_convert(*tq, *sp.tc, tl, st);
    if (!rc) rc = quirk_convert(*dq, *sp.dc, dl, st);
    if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "kv quirk");  // the bf16 copies go now
  }
  if (!rc)
    rc = cuda_check(lmx_launch(prefill_done_kernel, dim3((B + 127) / 128), dim3(128), 0, st, true, sp.s,
                               (const int32_t*)sp.prompts, P, (const int32_t*)sp.yprefill, tl, dl),
                    "prefill_done");
  if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "prefill");
  if (!rc) sp.prefilled = true;
  sp.it_rp.assign(B, 0);
  sp.it_em.assign(B, 0);
  sp.it_buf.assign((size_t)B * sp.cfg.max_tokens, 0);
  return rc;
}

// Decode until every sequence has max_tokens: one captured graph per step.
// Capture one speculative step as a CUDA graph (once per decoder).
static int spec_capture(Spec& sp) {
  if (sp.exec) return LMX_OK;
  cudaStream_t st = sp.st;
  int rc = cuda_check(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "capture begin");
  if (rc) return rc;
  int rc2 = spec_step(sp);
  cudaGraph_t g = nullptr;
  rc = cuda_check(cudaStreamEndCapture(st, &g), "capture end");
  if (rc2) {
    if (g) cudaGraphDestroy(g);
    return rc2;
  }
  if (rc) return rc;
  sp.graph = g;
  return cuda_check(cudaGraphInstantiate(&sp.exec, g, 0), "graph instantiate");
}

static int spec_decode(Spec& sp, int use_graph, double* seconds) {
  if (!sp.prefilled) return set_error(LMX_ERR_INVALID, "spec: decode before prefill");
  cudaStream_t st = sp.st;
  int rc = LMX_OK;
  if (use_graph) rc = spec_capture(sp);
  if (rc) return rc;
  const int B = sp.cfg.batch, MT = sp.cfg.max_tokens;
  std::vector<int> em(B);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, st);
  const int check_every = 4;
  sp.replays = 0;
  for (int it = 0; it < MT + 1 && !rc; it += check_every) {
    for (int k = 0; k < check_every && !rc; ++k, ++sp.replays)
      rc = use_graph ? cuda_check(cudaGraphLaunch(sp.exec, st), "graph launch") : spec_step(sp);
    if (rc) break;
    rc = cuda_check(cudaMemcpyAsync(em.data(), sp.s.emitted, B * 4, cudaMemcpyDeviceToHost, st), "emitted");
    if (!rc) rc = cuda_check(cudaStreamSynchronize(st), "decode step");
    bool all = true;
    for (int b = 0; b < B; ++b) all = all && em[b] >= MT;
    if (all) break;
  }
  cudaEventRecord(e1, st);
  cudaEventSynchronize(e1);
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (seconds) *seconds = ms * 1e-3;
  if (!rc) {
    unsigned code = 0;
    cudaMemcpyFromSymbol(&code, g_lmx_kernel_error, sizeof(code));
    if (code) rc = set_error(LMX_ERR_CUDA, "kernel reported error 0x%x", code);
  }
  return rc;
}

// TokenIterator::next() (src/common/generate.cpp:968-1045): the next token of
// every sequence in emission order (d0 first, then the accepted drafts; the
// correction / bonus token is the next step's d0).  One speculative step (one
// graph replay; K = 0: one plain decode step, generate.cpp:671-686) runs only
// when a sequence that has not reached max_tokens has no token left to read.
// tok[b] = -1 once sequence b has given all max_tokens; *n_live counts the
// others (0 is the reference's nullopt).
static int spec_next(Spec& sp, int32_t* tok, int* n_live) {
  if (!sp.prefilled) return set_error(LMX_ERR_INVALID, "spec_next: before prefill");
  const int B = sp.cfg.batch, MT = sp.cfg.max_tokens;
  int rc = spec_capture(sp);
  bool need = false;
  for (int b = 0; b < B; ++b) need = need || (sp.it_rp[b] < MT && sp.it_rp[b] >= sp.it_em[b]);
  if (!rc && need) {
    rc = cuda_check(cudaGraphLaunch(sp.exec, sp.st), "graph launch");
    ++sp.replays;
    if (!rc)
      rc = cuda_check(cudaMemcpyAsync(sp.it_em.data(), sp.s.emitted, (size_t)B * 4, cudaMemcpyDeviceToHost, sp.st),
                      "emitted");
    if (!rc)
      rc = cuda_check(cudaMemcpyAsync(sp.it_buf.data(), sp.s.out, sp.it_buf.size() * 4, cudaMemcpyDeviceToHost,
                                      sp.st),
                      "stream");
    if (!rc) rc = cuda_check(cudaStreamSynchronize(sp.st), "spec_next");
    if (!rc) {
      unsigned code = 0;
      cudaMemcpyFromSymbol(&code, g_lmx_kernel_error, sizeof(code));
      if (code) rc = set_error(LMX_ERR_CUDA, "kernel reported error 0x%x", code);
    }
  }
  if (rc) return rc;
  int live = 0;
  for (int b = 0; b < B; ++b) {
    if (sp.it_rp[b] < std::min(sp.it_em[b], MT)) {
      tok[b] = sp.it_buf[(size_t)b * MT + sp.it_rp[b]++];
      ++live;
    } else {
      tok[b] = -1;
    }
  }
  *n_live = live;
  return LMX_OK;
}

// generate() (src/common/generate.cpp:1061-1125) per sequence: prefill the
// prompts, then tokens from spec_next until every sequence has stopped.  The
// cancellation predicate is polled before every step (generate.h:218-228);
// a token in eos_ids ends its sequence without being counted or passed on;
// on_token returning nonzero ends its sequence after it (GenerateDisposition::
// stop).  Timings as GenerateCompletionInfo (generate.h:170-199): prompt_time
// the prefill's wall time, generation_time from a sequence's first token to
// its end (the reference restarts its clock at the first token).
static int spec_generate(Spec& sp, const int32_t* prompts, const int32_t* eos, int n_eos, lmx_cancel_fn cancel,
                         void* cancel_user, lmx_token_fn on_token, void* token_user, lmx_completion_info* info) {
  using clk = std::chrono::steady_clock;
  const int B = sp.cfg.batch;
  const auto t0 = clk::now();
  int rc = spec_prefill(sp, prompts);
  if (rc) return rc;
  const double prompt_s = std::chrono::duration<double>(clk::now() - t0).count();
  std::vector<int> count(B, 0);
  std::vector<char> done(B, 0), started(B, 0);
  std::vector<clk::time_point> first(B, clk::now()), end(B, clk::now());
  std::vector<int32_t> tok(B);
  for (;;) {
    if (cancel && cancel(cancel_user)) break;
    int live = 0;
    rc = spec_next(sp, tok.data(), &live);
    if (rc) return rc;
    if (!live) break;
    bool any = false;
    for (int b = 0; b < B; ++b) {
      if (done[b] || tok[b] < 0) continue;
      if (!started[b]) {
        started[b] = 1;
        first[b] = clk::now();
      }
      bool is_eos = false;
      for (int i = 0; i < n_eos && !is_eos; ++i) is_eos = eos[i] == tok[b];
      if (is_eos) {
        done[b] = 1;
        end[b] = clk::now();
        continue;
      }
      ++count[b];
      if (on_token && on_token(token_user, b, tok[b])) {
        done[b] = 1;
        end[b] = clk::now();
        continue;
      }
      any = true;
    }
    bool all = true;
    for (int b = 0; b < B; ++b) all = all && (done[b] || sp.it_rp[b] >= sp.cfg.max_tokens);
    if (all || !any) {
      bool pending = false;  // a sequence may still have tokens to read
      for (int b = 0; b < B; ++b) pending = pending || (!done[b] && sp.it_rp[b] < sp.cfg.max_tokens);
      if (!pending) break;
    }
  }
  std::vector<int> steps(B), acc(B);
  rc = cuda_check(cudaMemcpy(steps.data(), sp.s.steps, (size_t)B * 4, cudaMemcpyDeviceToHost), "stats");
  if (!rc) rc = cuda_check(cudaMemcpy(acc.data(), sp.s.accepted, (size_t)B * 4, cudaMemcpyDeviceToHost), "stats");
  if (rc) return rc;
  const auto now = clk::now();
  for (int b = 0; b < B && info; ++b) {
    lmx_completion_info& f = info[b];
    f.prompt_token_count = sp.cfg.prompt_len;
    f.generation_token_count = count[b];
    f.prompt_time = prompt_s;
    f.generation_time = started[b] ? std::chrono::duration<double>((done[b] ? end[b] : now) - first[b]).count() : 0.0;
    f.mtp_draft_tokens_proposed = steps[b] * sp.cfg.K;
    f.mtp_draft_tokens_accepted = acc[b];
    f.mtp_speculative_steps = steps[b];
  }
  return LMX_OK;
}

}  // namespace lmx

// ---------------------------------------------------------------------------
// C ABI: models, caches, forward, speculative generation
// ---------------------------------------------------------------------------
using namespace lmx;

extern "C" int lmx_set_device(int device) { return cuda_check(cudaSetDevice(device), "set_device"); }

extern "C" int lmx_set_fused_decode(int on) {
  if (on != 0 && on != 1) return set_error(LMX_ERR_INVALID, "fused_decode: 0 or 1");
  g_fused_decode = on;
  return LMX_OK;
}
extern "C" int lmx_fused_decode(void) { return g_fused_decode; }

extern "C" int lmx_set_sdpa_tc_min_cache(int rows) {
  if (rows < 0) return set_error(LMX_ERR_INVALID, "sdpa_tc_min_cache: rows >= 0 (0 = only by row count)");
  g_sdpa_long_cache = rows;
  return LMX_OK;
}
extern "C" int lmx_sdpa_tc_min_cache(void) { return g_sdpa_long_cache; }

extern "C" int lmx_model_create(const lmx_model_config* cfg, uint64_t seed, void** model) {
  if (!cfg || !model) return set_error(LMX_ERR_INVALID, "model_create: null argument");
  Model* m = nullptr;
  int rc = model_create(*cfg, seed, nullptr, &m);
  if (!rc) *model = m;
  return rc;
}

extern "C" int lmx_model_create_tp(const lmx_model_config* cfg, uint64_t seed, void* comm, void** model) {
  if (!cfg || !model) return set_error(LMX_ERR_INVALID, "model_create_tp: null argument");
  Model* m = nullptr;
  int rc = model_create(*cfg, seed, (TpComm*)comm, &m);
  if (!rc) *model = m;
  return rc;
}

extern "C" int lmx_tp_comm_create(int rank, int size, int max_rows, int max_hidden, void** comm) {
  if (!comm) return set_error(LMX_ERR_INVALID, "tp_comm_create: null argument");
  TpComm* c = nullptr;
  int rc = tp_comm_create(rank, size, max_rows, max_hidden, &c);
  if (!rc) *comm = c;
  return rc;
}

extern "C" int lmx_tp_comm_handle(void* comm, void* handle) {
  TpComm* c = (TpComm*)comm;
  if (!c || !handle) return set_error(LMX_ERR_INVALID, "tp_comm_handle: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == LMX_TP_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  int rc = cuda_check(cudaIpcGetMemHandle(&h, c->block), "tp_comm_handle");
  if (!rc) std::memcpy(handle, &h, sizeof(h));
  return rc;
}

extern "C" int lmx_tp_comm_open(void* comm, const void* handles) {
  TpComm* c = (TpComm*)comm;
  if (!c || !handles) return set_error(LMX_ERR_INVALID, "tp_comm_open: null argument");
  return tp_comm_open(*c, handles);
}

extern "C" int lmx_tp_comm_free(void* comm) {
  delete (TpComm*)comm;
  return LMX_OK;
}

extern "C" size_t lmx_tp_comm_block_bytes(void* comm) { return comm ? ((TpComm*)comm)->block_bytes : 0; }

extern "C" int lmx_tp_comm_attach(void* comm, int peer, void* peer_block) {
  TpComm* c = (TpComm*)comm;
  if (!c) return set_error(LMX_ERR_INVALID, "tp_comm_attach: null comm");
  return tp_comm_attach(*c, peer, peer_block);
}

extern "C" int lmx_tp_comm_partial(void* comm, void** partial) {
  TpComm* c = (TpComm*)comm;
  if (!c || !partial) return set_error(LMX_ERR_INVALID, "tp_comm_partial: null argument");
  *partial = tp_slot(*c, c->sel);
  return LMX_OK;
}

extern "C" int lmx_tp_allreduce_rmsnorm(void* comm, const void* partial, int rows, int hidden, void* h,
                                        const void* norm_w, float eps, void* xn, void* stream) {
  TpComm* c = (TpComm*)comm;
  if (!c || !h || !norm_w || !xn || rows < 1 || hidden < 8 || hidden % 8)
    return set_error(LMX_ERR_INVALID, "tp_allreduce_rmsnorm: bad arguments");
  if (!c->opened) return set_error(LMX_ERR_INVALID, "tp_allreduce_rmsnorm: comm not open");
  if (rows > c->max_rows || hidden > c->max_hidden)
    return set_error(LMX_ERR_INVALID, "tp_allreduce_rmsnorm: %dx%d exceeds the comm", rows, hidden);
  cudaStream_t st = (cudaStream_t)stream;
  bf16_t* slot = tp_slot(*c, c->sel);
  int rc = LMX_OK;
  if (partial && partial != slot)
    rc = cuda_check(cudaMemcpyAsync(slot, partial, (size_t)rows * hidden * 2, cudaMemcpyDeviceToDevice, st),
                    "tp_allreduce_rmsnorm: stage partial");
  if (!rc)
    rc = launch_tp_allreduce_norm(*c, c->sel, rows, hidden, (bf16_t*)h, (const bf16_t*)norm_w, eps, (bf16_t*)xn,
                                  st);
  if (!rc) c->sel ^= 1;
  return rc;
}

extern "C" int lmx_model_view(void* model, int n_layers, void** view) {
  Model* m = (Model*)model;
  if (!m || !view || n_layers < 1 || n_layers > m->n_layers)
    return set_error(LMX_ERR_INVALID, "model_view: bad arguments");
  Model* v = new Model(*m);
  v->n_layers = n_layers;
  *view = v;
  return LMX_OK;
}

extern "C" int lmx_model_free(void* model) {
  delete (Model*)model;
  return LMX_OK;
}

extern "C" int lmx_model_weight(void* model, int layer, int kind, void* w_host, void* s_host,
                                void* b_host) {
  Model* m = (Model*)model;
  if (!m) return set_error(LMX_ERR_INVALID, "model_weight: null model");
  const QWeight* q = nullptr;
  if (kind == 7) q = &m->embed;
  else if (kind == 8) q = &m->head();
  else if (layer >= 0 && layer < (int)m->L.size() && kind >= 0 && kind < 7) q = &m->L[layer].w[kind];
  if (!q) return set_error(LMX_ERR_INVALID, "model_weight: bad layer/kind");
  const size_t nw = (size_t)q->N * q->K * q->bits / 32, ng = (size_t)q->N * (q->K / 64);
  int rc = cuda_check(cudaMemcpy(w_host, q->w, nw * 4, cudaMemcpyDeviceToHost), "copy w");
  if (!rc) rc = cuda_check(cudaMemcpy(s_host, q->s, ng * 2, cudaMemcpyDeviceToHost), "copy s");
  if (!rc) rc = cuda_check(cudaMemcpy(b_host, q->b, ng * 2, cudaMemcpyDeviceToHost), "copy b");
  return rc;
}

struct CacheHandle {
  Cache* c = nullptr;
  Workspace ws;
  int Tmax = 0;
  ~CacheHandle() { delete c; }
};

extern "C" int lmx_cache_create(void* model, int n_layers, int batch, int capacity, int kv_bits,
                                int max_tokens_per_forward, void** cache) {
  Model* m = (Model*)model;
  if (!m || !cache || max_tokens_per_forward < 1) return set_error(LMX_ERR_INVALID, "cache_create: bad arguments");
  auto h = std::make_unique<CacheHandle>();
  int rc = cache_create(*m, n_layers, batch, capacity, kv_bits, &h->c);
  if (!rc) rc = workspace_create(*m, batch, max_tokens_per_forward, capacity, batch * max_tokens_per_forward, h->ws);
  if (!rc) rc = dec_ws_reserve(h->ws, *m, kDecMaxRows);
  if (rc) return rc;
  h->Tmax = max_tokens_per_forward;
  *cache = h.release();
  return LMX_OK;
}

extern "C" int lmx_cache_free(void* cache) {
  delete (CacheHandle*)cache;
  return LMX_OK;
}

// KVCache::set_position (src/common/kv_cache.cpp:135-142): rows past pos are dropped.
extern "C" int lmx_cache_set_position(void* cache, int seq, int pos) {
  CacheHandle* h = (CacheHandle*)cache;
  if (!h || seq < 0 || seq >= h->c->B) return set_error(LMX_ERR_INVALID, "set_position: bad sequence");
  int cur = 0;
  int rc = cuda_check(cudaMemcpy(&cur, h->c->len + seq, 4, cudaMemcpyDeviceToHost), "len");
  if (!rc && pos < cur) rc = cuda_check(cudaMemcpy(h->c->len + seq, &pos, 4, cudaMemcpyHostToDevice), "len");
  return rc;
}

extern "C" int lmx_cache_fill_synthetic(void* cache, int rows, uint64_t seed, uint32_t tid_base) {
  CacheHandle* h = (CacheHandle*)cache;
  if (!h) return set_error(LMX_ERR_INVALID, "fill_synthetic: null cache");
  return cache_fill_synthetic(*h->c, rows, seed, tid_base, 0);
}

extern "C" int lmx_cache_len(void* cache, int seq, int* len) {
  CacheHandle* h = (CacheHandle*)cache;
  if (!h || !len || seq < 0 || seq >= h->c->B) return set_error(LMX_ERR_INVALID, "cache_len: bad arguments");
  return cuda_check(cudaMemcpy(len, h->c->len + seq, 4, cudaMemcpyDeviceToHost), "len");
}

// One forward of tokens [B, T] (host) through the first n_layers; logits
// [B, T, V] bf16 copied to logits_host (may be NULL).  Advances the lengths.
extern "C" int lmx_forward(void* model, void* cache, int n_layers, const int32_t* tokens_host, int B, int T,
                           void* logits_host) {
  Model* m = (Model*)model;
  CacheHandle* h = (CacheHandle*)cache;
  if (!m || !h || !tokens_host || T < 1 || T > h->Tmax || B != h->c->B)
    return set_error(LMX_ERR_INVALID, "forward: bad arguments");
  int32_t* tok = nullptr;
  Arena ar;
  int rc = ar.alloc(&tok, (size_t)B * T);
  if (!rc) rc = cuda_check(cudaMemcpy(tok, tokens_host, (size_t)B * T * 4, cudaMemcpyHostToDevice), "tokens");
  if (!rc) rc = forward(*m, *h->c, n_layers, tok, T, 0, B, T, h->ws, logits_host ? h->ws.logits : nullptr, false, 0);
  if (!rc) rc = add_len(h->c->len, B, T, 0);
  if (!rc) rc = cuda_check(cudaDeviceSynchronize(), "forward");
  if (!rc && logits_host)
    rc = cuda_check(cudaMemcpy(logits_host, h->ws.logits, (size_t)B * T * m->vl * 2, cudaMemcpyDeviceToHost),
                    "logits");
  return rc;
}

extern "C" int lmx_spec_create(void* target, void* draft, int draft_layers, const lmx_spec_config* cfg,
                               void** spec) {
  Model* tm = (Model*)target;
  Model* dm = draft ? (Model*)draft : tm;
  if (!tm || !cfg || !spec) return set_error(LMX_ERR_INVALID, "spec_create: null argument");
  const int dl = draft_layers > 0 ? draft_layers : dm->n_layers;
  if (dl > dm->n_layers) return set_error(LMX_ERR_INVALID, "spec_create: draft_layers > draft layers");
  Spec* sp = nullptr;
  int rc = spec_create(tm, dm, dl, *cfg, &sp);
  if (!rc) *spec = sp;
  return rc;
}

extern "C" int lmx_spec_prefill(void* spec, const int32_t* prompts_host) {
  if (!spec || !prompts_host) return set_error(LMX_ERR_INVALID, "spec_prefill: null argument");
  return spec_prefill(*(Spec*)spec, prompts_host);
}

extern "C" int lmx_spec_decode(void* spec, int use_graph, double* seconds) {
  if (!spec) return set_error(LMX_ERR_INVALID, "spec_decode: null argument");
  return spec_decode(*(Spec*)spec, use_graph, seconds);
}

extern "C" int lmx_spec_result(void* spec, int32_t* out_host, int64_t* stats_host) {
  Spec* sp = (Spec*)spec;
  if (!sp) return set_error(LMX_ERR_INVALID, "spec_result: null argument");
  const int B = sp->cfg.batch;
  int rc = LMX_OK;
  if (out_host)
    rc = cuda_check(cudaMemcpy(out_host, sp->s.out, (size_t)B * sp->cfg.max_tokens * 4, cudaMemcpyDeviceToHost),
                    "out");
  if (!rc && stats_host) {
    std::vector<int> steps(B), acc(B), em(B);
    rc = cuda_check(cudaMemcpy(steps.data(), sp->s.steps, B * 4, cudaMemcpyDeviceToHost), "stats");
    if (!rc) rc = cuda_check(cudaMemcpy(acc.data(), sp->s.accepted, B * 4, cudaMemcpyDeviceToHost), "stats");
    if (!rc) rc = cuda_check(cudaMemcpy(em.data(), sp->s.emitted, B * 4, cudaMemcpyDeviceToHost), "stats");
    int64_t st = 0, ac = 0, e = 0;
    for (int b = 0; b < B; ++b) { st += steps[b]; ac += acc[b]; e += em[b]; }
    stats_host[0] = st;
    stats_host[1] = st * sp->cfg.K;
    stats_host[2] = ac;
    stats_host[3] = e;
    stats_host[4] = sp->replays;
  }
  return rc;
}

extern "C" int lmx_spec_next(void* spec, int32_t* tokens_host, int* n_live) {
  if (!spec || !tokens_host || !n_live) return set_error(LMX_ERR_INVALID, "spec_next: null argument");
  return spec_next(*(Spec*)spec, tokens_host, n_live);
}

extern "C" int lmx_spec_generate(void* spec, const int32_t* prompts_host, const int32_t* eos_ids, int n_eos,
                                 lmx_cancel_fn should_cancel, void* cancel_user, lmx_token_fn on_token,
                                 void* token_user, lmx_completion_info* info) {
  if (!spec || !prompts_host || n_eos < 0 || (n_eos > 0 && !eos_ids))
    return set_error(LMX_ERR_INVALID, "spec_generate: bad arguments");
  return spec_generate(*(Spec*)spec, prompts_host, eos_ids, n_eos, should_cancel, cancel_user, on_token, token_user,
                       info);
}

extern "C" int lmx_spec_free(void* spec) {
  delete (Spec*)spec;
  return LMX_OK;
}

namespace lmx {
// Algorithmic HBM bytes of one quantized matrix read plus its activations.
static double qmm_bytes(const QWeight& w, int M) {
  const int bits = w.bits;
  return (double)w.N * w.K * bits / 8 + (double)w.N * (w.K / 64) * 4 + (double)M * w.K * 2 + (double)M * w.N * 2;
}

// Time `what` on the spec's stream with CUDA events (iters launches, after the
// decode): 0 verify pass (target forward over K+1 tokens incl. lm_head),
// 1 one draft token (draft forward T=1 incl. lm_head), 2 lm_head at
// M = B(K+1), 3 lm_head at M = B.  bytes = algorithmic bytes per launch.
static int spec_profile(Spec& sp, int what, int iters, double* seconds, double* bytes) {
  if (!sp.prefilled) return set_error(LMX_ERR_INVALID, "profile before prefill");
  const int B = sp.cfg.batch, K = sp.cfg.K;
  cudaStream_t st = sp.st;
  std::vector<int> tl(B), dl(B);
  int rc = cuda_check(cudaMemcpy(tl.data(), sp.tc->len, B * 4, cudaMemcpyDeviceToHost), "len");
  if (!rc) rc = cuda_check(cudaMemcpy(dl.data(), sp.dc->len, B * 4, cudaMemcpyDeviceToHost), "len");
  if (rc) return rc;
  double by = 0;
  auto model_bytes = [&](const Model& m, int nl, int M, const std::vector<int>& lens, int T, bool head) {
    double s = 0;
    for (int l = 0; l < nl; ++l)
      for (int k = 0; k < 7; ++k) s += qmm_bytes(m.L[l].w[k], M);
    for (int b = 0; b < B; ++b)  // K and V rows read by attention, new rows written
      s += (double)nl * 2 * m.hk * (lens[b] + T) * kHeadDim * (sp.cfg.kv_bits == 16 ? 2.0 : sp.cfg.kv_bits / 8.0 + 4.0 / 64);
    if (head) s += qmm_bytes(m.head(), M);
    return s;
  };
  if (what == 1 && K == 0) return set_error(LMX_ERR_INVALID, "profile: no draft (K = 0)");
  if (what == 0) by = model_bytes(*sp.tm, sp.tm->n_layers, B * (K + 1), tl, K + 1, true);
  else if (what == 1) by = model_bytes(*sp.dm, sp.dl, B, dl, 1, true);
  else if (what == 2) by = qmm_bytes(sp.tm->head(), B * (K + 1));
  else if (what == 3) by = qmm_bytes(sp.tm->head(), B);
  else return set_error(LMX_ERR_INVALID, "profile: what=%d", what);
  auto once = [&]() -> int {
    if (what == 0)
      return forward(*sp.tm, *sp.tc, sp.tm->n_layers, sp.s.vt, K + 1, 0, B, K + 1, sp.ws, sp.ws.logits, false, st);
    if (what == 1)
      return forward(*sp.dm, *sp.dc, sp.dl, sp.s.drafts, K, 0, B, 1, sp.ws, sp.ws.logits, true, st);
    QmmCall hc;
    hc.M = what == 2 ? B * (K + 1) : B;
    hc.x = sp.ws.h;
    if (qmm_uses_mma(hc.M)) {  // the tcgen05 path takes normalised rows
      const int r2 = launch_rms_norm(sp.ws.h, sp.tm->final_norm, sp.ws.xn, hc.M, sp.tm->c.hidden, sp.tm->c.eps, st);
      if (r2) return r2;
      hc.x = sp.ws.xn;
    } else {
      hc.norm_w = sp.tm->final_norm;
    }
    hc.eps = sp.tm->c.eps;
    hc.mat[0] = sp.tm->head().mat();
    hc.N = sp.tm->vl;
    hc.y = sp.ws.logits;
    hc.ldy = sp.tm->vl;
    hc.K = sp.tm->c.hidden;
    hc.bits = sp.tm->head().bits;
    return launch_qmm(hc, st);
  };
  for (int i = 0; i < 3 && !rc; ++i) rc = once();
  // timed as the decode runs it: the pass captured into a CUDA graph and
  // replayed, so host launch costs do not enter the figure
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  if (!rc) rc = cuda_check(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "profile: capture");
  if (!rc) {
    const int rc_once = once();
    const int rc_end = cuda_check(cudaStreamEndCapture(st, &graph), "profile: capture end");
    rc = rc_once ? rc_once : rc_end;
  }
  if (!rc) rc = cuda_check(cudaGraphInstantiate(&exec, graph, 0), "profile: instantiate");
  if (!rc) rc = cuda_check(cudaGraphLaunch(exec, st), "profile: warm-up replay");
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, st);
  nvtxRangePushA(what == 0 ? "lmx_verify_pass" : (what == 1 ? "lmx_draft_token" : "lmx_lm_head"));
  for (int i = 0; i < iters && !rc; ++i) rc = cuda_check(cudaGraphLaunch(exec, st), "profile: replay");
  nvtxRangePop();
  cudaEventRecord(e1, st);
  if (!rc) rc = cuda_check(cudaEventSynchronize(e1), "profile");
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  if (seconds) *seconds = ms * 1e-3 / (iters > 0 ? iters : 1);
  if (bytes) *bytes = by;
  return rc;
}

// Kernel launches of one speculative step (the graph's node count).
static int spec_step_launches(Spec& sp, int64_t* n) {
  if (!sp.graph) return set_error(LMX_ERR_INVALID, "no graph captured yet");
  size_t nodes = 0;
  int rc = cuda_check(cudaGraphGetNodes(sp.graph, nullptr, &nodes), "graph nodes");
  *n = (int64_t)nodes;
  return rc;
}
}  // namespace lmx

extern "C" int lmx_spec_profile(void* spec, int what, int iters, double* seconds, double* bytes) {
  if (!spec) return set_error(LMX_ERR_INVALID, "spec_profile: null argument");
  return spec_profile(*(Spec*)spec, what, iters, seconds, bytes);
}

extern "C" int lmx_spec_step_launches(void* spec, int64_t* launches) {
  if (!spec || !launches) return set_error(LMX_ERR_INVALID, "spec_step_launches: null argument");
  return spec_step_launches(*(Spec*)spec, launches);
}

// ---------------------------------------------------------------------------
// C ABI: attention over a caller-described KV cache
// ---------------------------------------------------------------------------
namespace lmx {
static int kv_from_c(const lmx_kv* c, KvDesc& d) {
  if (!c || c->head_dim != kHeadDim || c->batch < 1 || c->kv_heads < 1 || c->capacity < 1 || !c->lengths)
    return set_error(LMX_ERR_INVALID, "lmx_kv: bad descriptor (head_dim must be 128)");
  std::memset(&d, 0, sizeof(d));
  d.B = c->batch;
  d.Hk = c->kv_heads;
  d.cap = c->capacity;
  d.bits = c->bits;
  d.len = c->lengths;
  if (c->bits == 16) {
    if (!c->k || !c->v || ((uintptr_t)c->k & 15) || ((uintptr_t)c->v & 15))
      return set_error(LMX_ERR_INVALID, "lmx_kv: k/v must be 16-byte aligned");
    d.k = (bf16_t*)c->k;
    d.v = (bf16_t*)c->v;
  } else if (c->bits == 4 || c->bits == 8) {
    if (!c->k_packed || !c->v_packed || !c->k_scales || !c->k_biases || !c->v_scales || !c->v_biases)
      return set_error(LMX_ERR_INVALID, "lmx_kv: packed cache pointers missing");
    if (((uintptr_t)c->k_packed | (uintptr_t)c->v_packed) & 15)
      return set_error(LMX_ERR_INVALID, "lmx_kv: packed k/v must be 16-byte aligned");
    d.kq = c->k_packed;
    d.vq = c->v_packed;
    d.ks = (bf16_t*)c->k_scales;
    d.kb = (bf16_t*)c->k_biases;
    d.vs = (bf16_t*)c->v_scales;
    d.vb = (bf16_t*)c->v_biases;
  } else {
    return set_error(LMX_ERR_UNSUPPORTED, "lmx_kv: bits %d", c->bits);
  }
  return LMX_OK;
}

static void sdpa_geometry(int T, int heads, int kv_heads, int capacity, int& tiles, int& splits) {
  const int G = heads / kv_heads;
  tiles = (G * T + kRowTile - 1) / kRowTile;
  splits = (capacity + kSplit - 1) / kSplit;
}

static size_t sdpa_scratch_bytes(int B, int T, int heads, int kv_heads, int capacity) {
  size_t pf = 0, nc = 0;
  sdpa_scratch_need(B, T, heads / kv_heads, kv_heads, capacity, pf, nc);
  return (pf * 4 + 255) / 256 * 256 + (nc * 4 + 255) / 256 * 256;
}

// Shared by lmx_sdpa_decode and its no-allocation variant: checks the shape
// and launches sdpa_split_kernel with the given scratch (partials first, then
// the counters).
static int sdpa_call(const void* q, const lmx_kv* kv, int T, int heads, float scale, void* scratch,
                     size_t scratch_bytes, void* out, cudaStream_t st) {
  KvDesc d;
  int rc = kv_from_c(kv, d);
  if (rc) return rc;
  if (!q || !out || T < 1 || heads < 1 || heads % d.Hk)
    return set_error(LMX_ERR_INVALID, "sdpa: bad shape");
  const size_t need = sdpa_scratch_bytes(d.B, T, heads, d.Hk, d.cap);
  if (!scratch || scratch_bytes < need)
    return set_error(LMX_ERR_INVALID, "sdpa: scratch needs %zu bytes", need);
  int tiles, splits;
  sdpa_geometry(T, heads, d.Hk, d.cap, tiles, splits);
  SdpaArgs sa;
  sa.q = (const bf16_t*)q;
  sa.kv = d;
  sa.T = T;
  sa.Hq = heads;
  sa.scale = scale;
  sa.nsplit = splits;
  sa.tiles = tiles;
  sa.part = (float*)scratch;
  sdpa_scratch_need(d.B, T, heads / d.Hk, d.Hk, d.cap, sa.part_floats, sa.n_counters);
  sa.counters = (unsigned*)((char*)scratch + (sa.part_floats * 4 + 255) / 256 * 256);
  sa.out = (bf16_t*)out;
  return launch_sdpa(sa, d.B, st);
}
}  // namespace lmx

namespace lmx {
// KV append over a caller-described cache: k_new / v_new bf16
// [batch][kv_heads][T][128] (the reference's update layout), row t of
// sequence b written at lengths[b] + t (quantized on append for 4/8-bit);
// one warp per (sequence, KV head, token, K or V).  A block past the
// capacity sets the device error word 0x42 and writes nothing.
__global__ void kv_append_kernel(KvDesc kv, const bf16_t* kn, const bf16_t* vn, int T, unsigned* err) {
  grid_wait();
  grid_launch_dependents();
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (int64_t)kv.B * kv.Hk * T * 2) return;
  const bool is_v = (w & 1) != 0;
  const int64_t r = w >> 1;  // ((b * Hk + h) * T + t)
  const int t = (int)(r % T);
  const int64_t bh = r / T;
  const int b = (int)(bh / kv.Hk);
  const int pos = kv.len[b] + t;
  if (kv.len[b] + T > kv.cap) {
    if (lane == 0 && t == 0) atomicExch(err, 0x42u);
    return;
  }
  float x[8];
  if (lane < 16) unpack8(*reinterpret_cast<const uint4*>((is_v ? vn : kn) + (size_t)r * kHeadDim + 8 * lane), x);
  else
    for (int e = 0; e < 8; ++e) x[e] = 0.0f;
  uint4 deq;
  dec_append(kv, !is_v, (size_t)bh * kv.cap + pos, lane, x, deq);
}

__global__ void kv_advance_kernel(int* len, int B, int T, int cap) {
  grid_wait();
  grid_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B && len[b] + T <= cap) len[b] += T;  // a refused block leaves the length
}

__global__ void kv_set_position_kernel(int* len, int seq, int pos) {
  grid_wait();
  grid_launch_dependents();
  if (threadIdx.x == 0 && pos < len[seq]) len[seq] = pos;
}
}  // namespace lmx

extern "C" int lmx_cache_kv(void* cache, int layer, lmx_kv* out) {
  CacheHandle* h = (CacheHandle*)cache;
  if (!h || !out || layer < 0 || layer >= h->c->n_layers) return set_error(LMX_ERR_INVALID, "cache_kv: bad arguments");
  const KvDesc& d = h->c->kv[layer];
  std::memset(out, 0, sizeof(*out));
  out->batch = d.B;
  out->kv_heads = d.Hk;
  out->head_dim = kHeadDim;
  out->capacity = d.cap;
  out->bits = d.bits;
  out->k = d.k;
  out->v = d.v;
  out->k_packed = d.kq;
  out->v_packed = d.vq;
  out->k_scales = d.ks;
  out->k_biases = d.kb;
  out->v_scales = d.vs;
  out->v_biases = d.vb;
  out->lengths = d.len;
  return LMX_OK;
}

extern "C" int lmx_kv_append(const lmx_kv* kv, const void* k_new, const void* v_new, int T, void* stream) {
  KvDesc d;
  int rc = kv_from_c(kv, d);
  if (rc) return rc;
  if (!k_new || !v_new || T < 1 || ((uintptr_t)k_new & 15) || ((uintptr_t)v_new & 15))
    return set_error(LMX_ERR_INVALID, "kv_append: bad block (16-byte aligned bf16 [batch][kv_heads][T][128])");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t threads = (int64_t)d.B * d.Hk * T * 2 * 32;
  rc = cuda_check(lmx_launch(kv_append_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, true, d,
                             (const bf16_t*)k_new, (const bf16_t*)v_new, T, device_error_word()),
                  "kv_append");
  if (!rc)
    rc = cuda_check(lmx_launch(kv_advance_kernel, dim3((d.B + 127) / 128), dim3(128), 0, st, true, d.len, d.B, T, d.cap),
                    "kv_append: lengths");
  return rc;
}

extern "C" int lmx_kv_set_position(const lmx_kv* kv, int seq, int pos, void* stream) {
  if (!kv || !kv->lengths || seq < 0 || seq >= kv->batch || pos < 0)
    return set_error(LMX_ERR_INVALID, "kv_set_position: bad arguments");
  return cuda_check(lmx_launch(kv_set_position_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, true,
                               (int*)kv->lengths, seq, pos),
                    "kv_set_position");
}

extern "C" size_t lmx_sdpa_scratch_bytes(int batch, int T, int heads, int kv_heads, int capacity) {
  if (batch < 1 || T < 1 || heads < 1 || kv_heads < 1 || capacity < 1 || heads % kv_heads) return 0;
  return sdpa_scratch_bytes(batch, T, heads, kv_heads, capacity);
}

extern "C" int lmx_sdpa_decode(const void* q, const lmx_kv* kv, int T, int heads, float scale, void* scratch,
                               size_t scratch_bytes, void* out, void* stream) {
  return sdpa_call(q, kv, T, heads, scale, scratch, scratch_bytes, out, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// C ABI: sampling and speculative acceptance with caller uniforms
// ---------------------------------------------------------------------------
extern "C" int lmx_sample(const void* logits, int rows, int V, float temperature, float top_p,
                          const uint32_t* u24, int32_t* out, void* stream) {
  if (rows == 0) return LMX_OK;
  if (!logits || !out || rows < 0 || V < 1) return set_error(LMX_ERR_INVALID, "sample: bad arguments");
  if (!(temperature > 0.0f)) return launch_argmax((const bf16_t*)logits, rows, V, out, (cudaStream_t)stream);
  if (!u24) return set_error(LMX_ERR_INVALID, "sample: uniforms required when temperature > 0");
  return cuda_check(samp_launch(sample_u_kernel, rows, V, 1, (cudaStream_t)stream,
                               (const bf16_t*)logits, V, temperature, top_p, u24, out),
                    "sample");
}

extern "C" int lmx_spec_accept(const void* target_logits, const void* draft_logits, const int32_t* drafts, int B,
                               int K, int V, float temperature, float top_p, const uint32_t* u_accept,
                               const uint32_t* u_final, int32_t* n_accepted, int32_t* out_tokens, void* stream) {
  if (B == 0) return LMX_OK;
  if (!target_logits || !drafts || !n_accepted || !out_tokens || B < 0 || K < 1 || V < 1)
    return set_error(LMX_ERR_INVALID, "spec_accept: bad arguments");
  if (!(temperature > 0.0f))
    return set_error(LMX_ERR_INVALID, "spec_accept: greedy acceptance runs inside lmx_spec_decode");
  if (!draft_logits || !u_accept || !u_final) return set_error(LMX_ERR_INVALID, "spec_accept: null argument");
  return cuda_check(samp_launch(accept_u_kernel, B, V, 2, (cudaStream_t)stream,
                               (const bf16_t*)target_logits, (const bf16_t*)draft_logits, drafts, K, V, temperature,
                               top_p, u_accept, u_final, n_accepted, out_tokens),
                    "spec_accept");
}
