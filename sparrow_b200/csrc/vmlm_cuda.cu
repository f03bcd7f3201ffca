// vmlm_cuda.cu -- host side of the C ABI declared in include/vmlm_cuda.h:
// device contexts, workspace, the weight registry, argument checks, kernel
// selection and launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/vmlm_cuda.h"
#include "prep.cuh"
#include "probe.cuh"
#include "decode.cuh"
#include "decode_sk.cuh"
#include "tc2_gemm.cuh"
#include "tc_gemm.cuh"
#include "variants.cuh"
#include "vmb_pool.cuh"
#include "vm_ops.cuh"

using namespace vmlm;

namespace {

thread_local std::string g_err;
std::recursive_mutex g_mu;
std::atomic<uint64_t> g_launches{0};

// Allocation-free Q8 entry point (end of this file): whether its scratch is set
// up on a device, and its device error word, read and cleared by vmlm_sync.
bool na_ready(int dev);
int na_take_error(int dev, int* code);

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define VMLM_CUDA(x)                                                                                    \
  do {                                                                                                  \
    cudaError_t e_ = (x);                                                                               \
    if (e_ != cudaSuccess)                                                                              \
      return fail(e_ == cudaErrorMemoryAllocation ? VMLM_ERR_OOM : VMLM_ERR_CUDA, "%s: %s (%s:%d)", #x, \
                  cudaGetErrorString(e_), __FILE__, __LINE__);                                          \
  } while (0)

#define VMLM_TRY(x)              \
  do {                           \
    int r_ = (x);                \
    if (r_ != VMLM_OK) return r_; \
  } while (0)

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
};

// Grow-only device buffer. Growing frees the old buffer (cudaFree waits for
// the device), so a call that needs more workspace than any earlier call
// cannot be captured into a CUDA graph.
int ensure(DevBuf& b, size_t bytes) {
  if (bytes == 0) bytes = 16;
  if (b.bytes >= bytes) return VMLM_OK;
  size_t nb = b.bytes * 2 > bytes ? b.bytes * 2 : bytes;
  nb = (nb + 255) & ~static_cast<size_t>(255);
  if (b.p) VMLM_CUDA(cudaFree(b.p));
  b.p = nullptr;
  b.bytes = 0;
  VMLM_CUDA(cudaMalloc(&b.p, nb));
  b.bytes = nb;
  return VMLM_OK;
}

// ensure() for buffers whose kernels expect zeros (split-tile slots and
// counters, flag words): a newly allocated buffer is cleared on `st`, the
// stream of the call that is about to use it, so the clear is ordered before
// that call's kernels whichever stream (library, caller's, non-blocking) it is.
int ensure_zeroed(DevBuf& b, size_t bytes, cudaStream_t st) {
  const size_t had = b.bytes;
  VMLM_TRY(ensure(b, bytes));
  if (b.bytes != had) VMLM_CUDA(cudaMemsetAsync(b.p, 0, b.bytes, st));
  return VMLM_OK;
}

constexpr int kCeMaxChunks = 8;           // GEMM row chunks of a copy-engine-gathered sharded call
constexpr double kCeMinPeerBytes = 16e6;  // peer bytes per call from which the copy engines carry the gather

struct Ctx {
  int dev = -1;
  int sms = 0;
  cudaStream_t stream = nullptr;
  DevBuf act;       // digit planes / split terms
  DevBuf small;     // exps | nonfinite | term_flags, each [M] int
  DevBuf slots;     // swap-mode split-tile accumulators (zeroed once, self-clearing)
  DevBuf counters;  // split-tile counters (zeroed once, self-resetting)
  DevBuf shard_done;  // row-sharded calls: CTA completion counter (zeroed once, self-resetting)
  DevBuf sync;      // prep completion counter and term-flag OR (zeroed once, self-resetting)
  // bf16 normal mode: term planes and per-row dirty bits of their own (zeroed
  // whenever the layout changes), and two term-flag words used by alternate calls
  DevBuf norm_terms, norm_dirty, norm_flags;
  int norm_m = -1, norm_kp = -1;
  unsigned norm_parity = 0;
  // f32 GEMM: term planes, dirty bits and NaN/Inf flags of both operands, and
  // their term-flag words (two per operand, used by alternate calls)
  DevBuf f32_ta, f32_tb, f32_da, f32_db, f32_nfa, f32_nfb, f32_flags;
  DevBuf f32_nft;            // NN calls: B's NaN/Inf column flags, two arrays used by alternate calls
  unsigned f32_nft_par = 0;
  int f32_m = -1, f32_n = -1, f32_kp = -1;
  bool f32_b_from_t = false;  // B's planes were last written by the transposing kernel
  unsigned f32_parity = 0;
  int* err = nullptr;       // device error word
  int* err_host = nullptr;  // pinned copy read after host-API calls
  DevBuf h_a, h_c, h_w, h_s, h_acc, h_b, h_g;  // host-API staging
  DevBuf xn;  // RMSNorm-fused Q8 calls: the normalised activations [M][K]
  DevBuf grp_planes;  // grouped Q8 batches in planes mode: every problem's planes, exponents and flags
  // host-pointer calls pipelined by row chunks: copies in and out on streams of
  // their own, ordered against the compute stream by events
  cudaStream_t s_in = nullptr, s_out = nullptr;
  // row-sharded calls gathered by copy engines: one stream per peer, events
  // for the chunks of the GEMM and for each peer stream's last copy
  cudaStream_t peer_st[kMaxPeers] = {};
  cudaEvent_t chunk_ev[kCeMaxChunks] = {};
  cudaEvent_t peer_done[kMaxPeers] = {};
  // row-sharded calls on more than two GPUs: the push kernels' stream
  cudaStream_t push_st = nullptr;
  cudaEvent_t push_done = nullptr;
  std::vector<cudaEvent_t> pipe_ev;
  bool attrs_set = false;
  std::map<std::pair<int, uint32_t>, int> dec_clusters;  // (cluster size, smem) -> co-resident clusters
};

std::map<int, Ctx*> g_ctx;
int g_host_dev = -1;

// Optional timing of the tensor-core GEMM launches (diagnostics): a CUDA event
// pair on the launch stream around each launch, summed by vmlm_profile_take.
bool g_profile = false;
// Optional per-CTA phase timestamps of the tensor-core GEMM (diagnostics).
unsigned long long* g_trace = nullptr;
size_t g_trace_ctas = 0;
int g_trace_dev = -1;
struct ProfPair {
  cudaEvent_t a, b;
  int dev;
};
std::vector<ProfPair> g_prof_live, g_prof_free;

struct Reg {
  size_t bytes;
  void* dptr;
  int dev;
};
std::map<uintptr_t, Reg> g_reg;

// Row-sharded calls: calls made so far on each rank's own inbox word.
std::map<uintptr_t, unsigned> g_inbox_calls;

// Peer buffers opened from IPC handles: one mapping per handle, shared by
// every open of it, released when the last user closes.
struct IpcMap {
  void* base;
  int refs;
};
std::map<std::string, IpcMap> g_ipc;            // handle bytes -> mapping
std::map<uintptr_t, std::string> g_ipc_users;    // pointer handed out -> handle bytes

int load_encoder() {
  if (g_encode) return VMLM_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  VMLM_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess || !fn) return fail(VMLM_ERR_CUDA, "cuTensorMapEncodeTiled not available");
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return VMLM_OK;
}

template <int MB>
int set_int4_smem_attr() {
  const int bytes = kI4SmemFloats * 4;
  VMLM_CUDA(cudaFuncSetAttribute(int4gs_kernel<MB, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  VMLM_CUDA(cudaFuncSetAttribute(int4gs_kernel<MB, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return VMLM_OK;
}

int set_int4_smem_attrs() {
  VMLM_CUDA(cudaFuncSetAttribute(int4gs_dp4a_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kI4SmemFloats * 4));
  VMLM_CUDA(cudaFuncSetAttribute(int4gs_dp4a_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kI4SmemFloats * 4));
  VMLM_TRY(set_int4_smem_attr<1>());
  VMLM_TRY(set_int4_smem_attr<2>());
  VMLM_TRY(set_int4_smem_attr<4>());
  return set_int4_smem_attr<8>();
}

template <TcMode M>
int set_smem_attr() {
  VMLM_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
  return VMLM_OK;
}

int get_ctx(int dev, Ctx** out) {
  auto it = g_ctx.find(dev);
  if (it != g_ctx.end()) {
    *out = it->second;
    return VMLM_OK;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(VMLM_ERR_NO_DEVICE, "no CUDA device");
  if (dev < 0 || dev >= ndev) return fail(VMLM_ERR_ARG, "device %d out of range (%d devices)", dev, ndev);
  cudaDeviceProp prop;
  VMLM_CUDA(cudaGetDeviceProperties(&prop, dev));
  if (prop.major != 10)
    return fail(VMLM_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", dev, prop.major,
                prop.minor);
  int prev = -1;
  VMLM_CUDA(cudaGetDevice(&prev));
  VMLM_CUDA(cudaSetDevice(dev));
  VMLM_TRY(load_encoder());
  Ctx* c = new Ctx();
  c->dev = dev;
  c->sms = prop.multiProcessorCount;
  VMLM_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  VMLM_CUDA(cudaMalloc(&c->err, sizeof(int)));
  VMLM_CUDA(cudaMemset(c->err, 0, sizeof(int)));
  VMLM_CUDA(cudaHostAlloc(&c->err_host, sizeof(int), cudaHostAllocDefault));
  *c->err_host = 0;
  VMLM_TRY(set_smem_attr<TcMode::kQ8Swap>());
  VMLM_TRY(set_smem_attr<TcMode::kBf16Swap>());
  VMLM_TRY(set_smem_attr<TcMode::kBf16Norm>());
  VMLM_TRY(set_smem_attr<TcMode::kI8Norm>());
  VMLM_TRY(set_smem_attr<TcMode::kF32Norm>());
  VMLM_CUDA(cudaFuncSetAttribute(tc2_gemm_kernel<TcMode::kI8Norm>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kMaxSmem));
  VMLM_CUDA(cudaFuncSetAttribute(tc2_gemm_kernel<TcMode::kBf16Norm>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kMaxSmem));
  VMLM_CUDA(cudaFuncSetAttribute(tc2_gemm_kernel<TcMode::kQ8Swap>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kMaxSmem));
  VMLM_CUDA(cudaFuncSetAttribute(q8_decode_kernel<DecNoGroup>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
  VMLM_CUDA(cudaFuncSetAttribute(q8_decode_kernel<DecGroup>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
  VMLM_CUDA(cudaFuncSetAttribute(q8_decode_sk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
  VMLM_TRY(set_int4_smem_attrs());
  g_ctx[dev] = c;
  if (prev >= 0 && prev != dev) cudaSetDevice(prev);
  *out = c;
  return VMLM_OK;
}

int current_ctx(Ctx** out) {
  int dev = -1;
  VMLM_CUDA(cudaGetDevice(&dev));
  return get_ctx(dev, out);
}

int host_ctx(Ctx** out) {
  if (g_host_dev < 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    g_host_dev = dev;
  }
  VMLM_CUDA(cudaSetDevice(g_host_dev));
  return get_ctx(g_host_dev, out);
}

// ------------------------------------------------------------- launches

// Launch with optional programmatic dependent launch and an optional cluster
// of `cluster` CTAs along x (1 = no cluster).
template <typename... KArgs, typename... Args>
int launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, int cluster,
              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  VMLM_CUDA(cudaLaunchKernelEx(&cfg, kern, args...));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return VMLM_OK;
}

template <typename... KArgs, typename... Args>
int launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
  return launch_ex(kern, grid, block, smem, st, pdl, 1, args...);
}

int make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t rows,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows) {
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = g_encode(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(VMLM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, pitch %llu, box %u x %u",
                static_cast<int>(r), static_cast<unsigned long long>(inner), static_cast<unsigned long long>(rows),
                static_cast<unsigned long long>(row_bytes), box_inner, box_rows);
  return VMLM_OK;
}

// 3-D view (128-byte k-block, row, k-block index) of a row-major matrix whose
// row pitch is a whole number of 128-byte k-blocks; a box of box_rows rows x
// box_kb k-blocks lands as box_kb consecutive 128-byte-swizzled tiles
// (tma_load_3d). Rows and k-blocks past the matrix read as zeros.
int make_map3(CUtensorMap* m, CUtensorMapDataType dt, int esz, const void* base, uint64_t rows, uint64_t row_bytes,
              uint32_t box_rows, uint32_t box_kb) {
  if (row_bytes % 128 != 0) return fail(VMLM_ERR_SHAPE, "3-D tensor map needs whole 128-byte k-blocks per row");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(128 / esz), rows, row_bytes / 128};
  cuuint64_t strides[2] = {row_bytes, 128};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / esz), box_rows, box_kb};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(VMLM_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d): rows %llu, pitch %llu, box %u x %u",
                static_cast<int>(r), static_cast<unsigned long long>(rows), static_cast<unsigned long long>(row_bytes),
                box_rows, box_kb);
  return VMLM_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline long long cdiv(long long a, long long b) { return (a + b - 1) / b; }
inline int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

// Decode GEMMs with fewer tiles than a few waves split tiles between CTAs
// (stream-K) to keep every SM streaming weights; with more tiles, whole tiles
// round-robin lose little to the last partial wave and need no fixup.
bool use_streamk(const TcParams& p, int sms) {
  return static_cast<long long>(p.tiles_m) * p.tiles_n < 4ll * sms;
}

// Stage ring depth of the tcgen05 kernel for tile width bn (as many as fit).
int tc_stages(int bn) {
  int stages = 16;
  while (stages >= 2 && tc_smem_layout(stages, bn).total > static_cast<uint32_t>(kMaxSmem)) --stages;
  return stages;
}

// Co-resident clusters of `cl` CTAs of tc_gemm_kernel<MODE> at `smem` bytes.
template <TcMode MODE>
int tc_max_clusters(Ctx* ctx, int cl, uint32_t smem, int* out) {
  const auto key = std::make_pair(1000 + 16 * static_cast<int>(MODE) + cl, smem);
  auto it = ctx->dec_clusters.find(key);
  if (it != ctx->dec_clusters.end()) {
    *out = it->second;
    return VMLM_OK;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cl * ctx->sms));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cl);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  VMLM_CUDA(cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<MODE>, &cfg));
  ctx->dec_clusters[key] = n;
  *out = n;
  return VMLM_OK;
}

// Tile width and K split for a normal-mode GEMM (rows x N output, 128-row
// tiles). Each candidate is costed as waves x per-CTA time, the per-CTA time
// being the larger of its operand traffic at a per-SM L2 rate and its MMA work
// at a per-SM tensor rate derated for narrow tiles (narrow UMMA N runs the
// tensor pipe less efficiently), plus the split-tile reduction. A K split runs
// over a thread-block cluster (partials exchanged in distributed shared memory,
// summed in rank order), so it is used only when every cluster of the launch
// is co-resident.
struct NormPlan {
  int bn;
  int split;
};

template <TcMode MODE>
int plan_norm(Ctx* ctx, int rows, int N, int K, int esz, bool int_acc, NormPlan* out, double* t_out = nullptr) {
  const int cand[3] = {256, 128, 64};
  const double eff[3] = {1.0, 0.85, 0.5};
  const double l2_bps = 120e9;                             // per SM
  const double dsm_bps = 150e9;                            // per SM, distributed shared memory
  const double mac_ps = (int_acc ? 22e12 : 11e12) / 2.0;  // MACs per second per SM
  const int sms = ctx->sms;
  NormPlan best{256, 1};
  double best_t = 1e300;
  for (int i = 0; i < 3; ++i) {
    const long long tiles = cdiv(rows, kTileRows) * cdiv(N, cand[i]);
    const long long kb = cdiv(K, 128 / esz);
    for (int split = 1; split <= 4; split *= 2) {
      if (split > 1) {
        if (tiles * split > sms || split > kb) continue;
        int active = 0;
        VMLM_TRY(tc_max_clusters<MODE>(ctx, split, tc_smem_layout(tc_stages(cand[i]), cand[i]).total, &active));
        if (tiles > active) continue;
      }
      const double kk = static_cast<double>(K) / split;
      const double t_load = (kTileRows + cand[i]) * kk * esz / l2_bps;
      const double t_mma = static_cast<double>(kTileRows) * cand[i] * kk / (mac_ps * eff[i]);
      const double t_red =
          split > 1 ? (split - 1.0) / split * kTileRows * cand[i] * 4 / dsm_bps + 1.0e-6 : 0.0;
      const double waves = static_cast<double>(cdiv(tiles * split, sms));
      const double t = waves * ((t_load > t_mma ? t_load : t_mma) + t_red);
      if (t < best_t * 0.999) {
        best_t = t;
        best = NormPlan{cand[i], split};
      }
    }
  }
  *out = best;
  if (t_out) *t_out = best_t;
  return VMLM_OK;
}

// Diagnostics: an event pair around one GEMM launch (vmlm_profile_enable).
// Record a profiling event on st. Inside a stream capture the record becomes
// an event-record node of the graph (cudaEventRecordExternal), so the times
// can be read after the graph is replayed.
cudaError_t prof_record(cudaEvent_t e, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t r = cudaStreamIsCapturing(st, &cs);
  if (r != cudaSuccess) return r;
  return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(e, st, cudaEventRecordExternal)
                                             : cudaEventRecord(e, st);
}

int prof_begin(Ctx* c, cudaStream_t st, ProfPair* pp) {
  if (!g_prof_free.empty() && g_prof_free.back().dev == c->dev) {
    *pp = g_prof_free.back();
    g_prof_free.pop_back();
  } else {
    VMLM_CUDA(cudaEventCreate(&pp->a));
    VMLM_CUDA(cudaEventCreate(&pp->b));
    pp->dev = c->dev;
  }
  VMLM_CUDA(prof_record(pp->a, st));
  return VMLM_OK;
}

// The last profiled launch: kernel and plan, for vmlm_profile_kernel.
std::string g_prof_last;

const char* tc_mode_name(TcMode m) {
  switch (m) {
    case TcMode::kQ8Swap: return "kQ8Swap";
    case TcMode::kBf16Swap: return "kBf16Swap";
    case TcMode::kBf16Norm: return "kBf16Norm";
    case TcMode::kI8Norm: return "kI8Norm";
    case TcMode::kF32Norm: return "kF32Norm";
  }
  return "?";
}

int prof_end(cudaStream_t st, const ProfPair& pp, const std::string& what) {
  VMLM_CUDA(prof_record(pp.b, st));
  g_prof_live.push_back(pp);
  g_prof_last = what;
  return VMLM_OK;
}

// Plan and launch the tcgen05 kernel. units_min = tiles * k-blocks with one term.
template <TcMode MODE>
int run_tc(Ctx* c, cudaStream_t st, const CUtensorMap& ma, const CUtensorMap& mb, TcParams p, bool streamk,
           bool pdl, int split = 0) {
  const int stages = tc_stages(p.bn);
  if (stages < 2) return fail(VMLM_ERR_SHAPE, "tile too large for shared memory");
  p.stages = stages;
  p.tmem_cols = pow2_at_least(2 * p.bn);
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
  const long long units_min = tiles * p.kb_per_term;
  long long grid = streamk ? (units_min < c->sms ? units_min : c->sms) : (tiles < c->sms ? tiles : c->sms);
  constexpr bool kSwapMode = (MODE == TcMode::kQ8Swap || MODE == TcMode::kBf16Swap);
  p.csplit = 0;
  if (split > 1) {
    // an explicit K split: exactly `split` CTAs per tile (stream-K ranges with
    // grid = tiles * split); normal modes run it over a cluster of `split` CTAs
    while (split > p.kb_per_term) split >>= 1;
    grid = tiles * split;
    streamk = split > 1;
    if (!kSwapMode && split > 1) p.csplit = split;
  }
  if (grid < 1) grid = 1;
  p.streamk = streamk ? 1 : 0;
  if (streamk && kSwapMode) {
    VMLM_TRY(ensure_zeroed(c->slots, static_cast<size_t>(grid) * kTileRows * p.bn * 4, st));
    VMLM_TRY(ensure_zeroed(c->counters, static_cast<size_t>(tiles) * 4, st));
  }
  const int cluster = p.csplit > 1 ? p.csplit : 1;
  p.slots = static_cast<uint32_t*>(c->slots.p);
  p.counters = static_cast<int*>(c->counters.p);
  p.err = c->err;
  p.trace = (g_trace && g_trace_dev == c->dev && static_cast<size_t>(grid) <= g_trace_ctas) ? g_trace : nullptr;
  const TcSmem L = tc_smem_layout(stages, p.bn);
  if (!g_profile)
    return launch_ex(tc_gemm_kernel<MODE>, dim3(static_cast<unsigned>(grid)), dim3(kThreads), L.total, st, pdl,
                     cluster, ma, mb, p);
  ProfPair pp;
  VMLM_TRY(prof_begin(c, st, &pp));
  VMLM_TRY(launch_ex(tc_gemm_kernel<MODE>, dim3(static_cast<unsigned>(grid)), dim3(kThreads), L.total, st, false,
                     cluster, ma, mb, p));
  char what[160];
  snprintf(what, sizeof what, "tc_gemm_kernel<%s>: %d CTAs, tiles %d x %d (128 x %d), %s %d", tc_mode_name(MODE),
           static_cast<int>(grid), p.tiles_m, p.tiles_n, p.bn, p.csplit > 1 ? "cluster K split" : "stream-K",
           p.csplit > 1 ? p.csplit : p.streamk);
  return prof_end(st, pp, what);
}

// Large prefill GEMMs on CTA pairs (tc2_gemm_kernel): 256 x 256 tiles, one
// pair per cluster, persistent. Taken when there is at least about one pair
// tile per co-resident pair and no K split is planned.
constexpr int kPairBn = 256;

template <TcMode MODE>
int tc2_max_pairs(Ctx* ctx, uint32_t smem, int* out) {
  const auto key = std::make_pair(2000 + static_cast<int>(MODE), smem);
  auto it = ctx->dec_clusters.find(key);
  if (it != ctx->dec_clusters.end()) {
    *out = it->second;
    return VMLM_OK;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * ctx->sms));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  VMLM_CUDA(cudaOccupancyMaxActiveClusters(&n, tc2_gemm_kernel<MODE>, &cfg));
  ctx->dec_clusters[key] = n;
  *out = n;
  return VMLM_OK;
}

int tc2_stages(int bn, int kps = 1) {
  int stages = 16;
  while (stages >= 2 && tc2_smem_layout(stages, bn, kps).total > static_cast<uint32_t>(kMaxSmem)) --stages;
  return stages;
}

// k-blocks per stage of a CTA-pair launch. Several k-blocks per load (3-D
// maps) stream far faster than one (a 128-row x 128-byte 2-D box streams at
// about 5 TB/s from HBM and 32 GB/s per SM from L2; three k-blocks per load
// reach 6.5 TB/s and 84 GB/s per SM), so take 3, or 2, while three stages
// fit, else while two do (with two stages the MMA of a tensor-bound tile
// waits for each refill: C5 630 us with 2 k-blocks x 3 stages, 696 us with
// 3 x 2, 705 us with 1 x 6). 3-D maps need both operands' row pitches to be
// whole k-blocks.
int tc2_pick_kps(int bn, uint64_t a_row_bytes, uint64_t b_row_bytes) {
  if (a_row_bytes % 128 != 0 || b_row_bytes % 128 != 0) return 1;
  for (int min_stages = 3; min_stages >= 2; --min_stages)
    for (int kps = 3; kps >= 2; --kps)
      if (tc2_stages(bn, kps) >= min_stages) return kps;
  return 1;
}

bool use_pairs(const NormPlan& plan, long long rows, long long cols, int sms) {
  const long long pair_tiles = cdiv(rows, 2 * kTileRows) * cdiv(cols, kPairBn);
  return plan.split == 1 && rows >= 2 * kTileRows && pair_tiles * 5 >= static_cast<long long>(sms) * 2;
}

// p: a parameter set whose tiles_m / bn / maps the caller fills for pair
// tiles (A box 128 rows, B box bn / 2 rows), and ksplit (0 or 1: whole K;
// 2: kBf16Norm only, C zeroed before the launch).
template <TcMode MODE>
int run_tc2(Ctx* c, cudaStream_t st, const CUtensorMap& ma, const CUtensorMap& mb, TcParams p, bool pdl) {
  if (p.ksplit > 1 && (MODE != TcMode::kBf16Norm || p.ksplit > 2 || p.ksplit > p.kb_per_term))
    return fail(VMLM_ERR_SHAPE, "a K split of pair tiles takes bf16 calls, two ranges, a k-block each");
  if (p.kps < 1) p.kps = 1;
  p.stages = tc2_stages(p.bn, p.kps);
  if (p.stages < 2) return fail(VMLM_ERR_SHAPE, "pair tile too large for shared memory");
  p.tmem_cols = pow2_at_least(2 * p.bn);
  p.csplit = 0;
  p.streamk = 0;
  const Tc2Smem L = tc2_smem_layout(p.stages, p.bn, p.kps);
  int max_pairs = 0;
  VMLM_TRY(tc2_max_pairs<MODE>(c, L.total, &max_pairs));
  if (max_pairs < 1) return fail(VMLM_ERR_CUDA, "no CTA pair fits on this device");
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n * (p.ksplit > 1 ? p.ksplit : 1);
  const long long pairs = tiles < max_pairs ? tiles : max_pairs;
  p.err = c->err;
  p.trace = (g_trace && g_trace_dev == c->dev && static_cast<size_t>(2 * pairs) <= g_trace_ctas) ? g_trace : nullptr;
  if (!g_profile)
    return launch_ex(tc2_gemm_kernel<MODE>, dim3(static_cast<unsigned>(2 * pairs)), dim3(kThreads), L.total, st, pdl,
                     2, ma, mb, p);
  ProfPair pp;
  VMLM_TRY(prof_begin(c, st, &pp));
  VMLM_TRY(launch_ex(tc2_gemm_kernel<MODE>, dim3(static_cast<unsigned>(2 * pairs)), dim3(kThreads), L.total, st,
                     false, 2, ma, mb, p));
  char what[160];
  snprintf(what, sizeof what, "tc2_gemm_kernel<%s>: %d CTA pairs, tiles %d x %d (256 x %d), K ranges %d",
           tc_mode_name(MODE), static_cast<int>(pairs), p.tiles_m, p.tiles_n, p.bn, p.ksplit > 1 ? p.ksplit : 1);
  return prof_end(st, pp, what);
}

int check_dims(size_t m, size_t n, size_t k) {
  const size_t lim = static_cast<size_t>(1) << 31;
  if (m >= lim || n >= lim || k >= lim) return fail(VMLM_ERR_SHAPE, "m, n, k must each be < 2^31");
  return VMLM_OK;
}

// ------------------------------------------------------- Q8 decode path

// Cluster size and stage ring for the decode kernel, or c == 0 when the call
// does not fit it (more than 32 tokens, an x slice per CTA larger than one
// register batch, or more tiles than one wave of clusters: the persistent
// kernel streams those better).
struct DecPlan {
  int c = 0;
  int stages = 0;
  int kbr = 0;
  uint32_t smem = 0;
  int kps = 1;  // k-blocks per W stage (3-D maps when > 1)
};

// k-blocks per W stage of a decode CTA streaming ranges of about kbr k-blocks
// of rows of row_bytes: 3 (or 2, when that wastes fewer k-blocks at the end of
// a range) when rows are whole 128-byte k-blocks (3-D tensor maps), else 1.
int dec_pick_kps(long long row_bytes, int kbr) {
  if (row_bytes % 128 != 0 || kbr < 2) return 1;
  const int waste3 = static_cast<int>(cdiv(kbr, 3) * 3 - kbr), waste2 = static_cast<int>(cdiv(kbr, 2) * 2 - kbr);
  return waste2 < waste3 ? 2 : 3;
}

int max_active_clusters(Ctx* ctx, int cl, uint32_t smem, int* out) {
  const auto key = std::make_pair(cl, smem);
  auto it = ctx->dec_clusters.find(key);
  if (it != ctx->dec_clusters.end()) {
    *out = it->second;
    return VMLM_OK;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cl * ctx->sms));
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cl);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  VMLM_CUDA(cudaOccupancyMaxActiveClusters(&n, q8_decode_kernel<DecNoGroup>, &cfg));
  ctx->dec_clusters[key] = n;
  *out = n;
  return VMLM_OK;
}

int plan_decode(Ctx* ctx, int M, int N, int K, bool planes_mode, DecPlan* plan) {
  *plan = DecPlan{};
  if (M < 1 || M > kDecMaxTok) return VMLM_OK;
  const long long tiles = cdiv(N, kTileRows);
  const int kb = static_cast<int>(cdiv(K, kBlockBytes));
  const int rows_b = static_cast<int>(16 * cdiv(3 * M, 16));
  long long best_ctas = 0;
  for (int c = 1; c <= kDecMaxCluster && c <= kb; ++c) {
    const int kbr = static_cast<int>(cdiv(kb, c));
    // Making the planes here: a CTA's x slice must fit one register batch of
    // the plane warps; a second batch and the reloads of the digit pass queue
    // behind the weight stream (float4 chunks of x per k-block: kBlockBytes / 4).
    if (!planes_mode &&
        static_cast<long long>(M) * kbr * (kBlockBytes / 4) > static_cast<long long>(kDecRegChunks) * kDecEpiThreads)
      continue;
    const int kps = dec_pick_kps(K, kbr);
    const int ops = static_cast<int>(cdiv(kbr, kps));
    int stages = ops < 16 ? ops : 16;
    while (stages >= 1 && dec_smem_layout(stages, rows_b, kbr, M, c, kps).total > static_cast<uint32_t>(kMaxSmem))
      --stages;
    if (stages < 1 || (stages < 2 && ops > 1)) continue;
    const uint32_t smem = dec_smem_layout(stages, rows_b, kbr, M, c, kps).total;
    int active = 0;
    VMLM_TRY(max_active_clusters(ctx, c, smem, &active));
    if (tiles > active) continue;  // one wave only
    if (tiles * c > best_ctas) {
      best_ctas = tiles * c;
      *plan = DecPlan{c, stages, kbr, smem, kps};
    }
  }
  return VMLM_OK;
}

// planes != nullptr: planes mode (q8_planes_kernel's planes [3M][kp], exps, nonfinite).
int run_decode(Ctx* ctx, const float* a, const int8_t* q, const float* scale, float* out, int M, int N, int K,
               cudaStream_t st, const DecPlan& plan, const int8_t* planes = nullptr, int kp = 0,
               const int* exps = nullptr, const int* nonf = nullptr, long long ldo = 0) {
  DecParams p = {};
  p.n = N;
  p.k = K;
  p.m = M;
  p.kb = static_cast<int>(cdiv(K, kBlockBytes));
  p.cluster = plan.c;
  p.rows_b = static_cast<int>(16 * cdiv(3 * M, 16));
  p.kbr_max = plan.kbr;
  p.stages = plan.stages;
  p.kps = plan.kps;
  p.tmem_cols = pow2_at_least(p.rows_b);
  p.vec_x = (K % 4 == 0) && aligned16(a);
  p.x = a;
  p.ldx = K;
  p.w = q;
  p.scale = scale;
  p.out = out;
  p.ldo = ldo > 0 ? ldo : N;
  p.err = ctx->err;
  const long long grid = cdiv(N, kTileRows) * plan.c;
  p.trace = (g_trace && g_trace_dev == ctx->dev && static_cast<size_t>(grid) <= g_trace_ctas) ? g_trace : nullptr;
  p.planes_mode = planes ? 1 : 0;
  p.exps = exps;
  p.nonfinite = nonf;
  CUtensorMap mw, mp;
  if (p.kps > 1)
    VMLM_TRY(make_map3(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, N, K, kTileRows, p.kps));
  else
    VMLM_TRY(make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, K, N, K, 128, kTileRows));
  if (planes)
    VMLM_TRY(make_map(&mp, CU_TENSOR_MAP_DATA_TYPE_UINT8, planes, K, 3ull * M, kp, 128,
                      static_cast<uint32_t>(p.rows_b)));
  else
    mp = mw;  // unused
  ProfPair pp;
  if (g_profile) VMLM_TRY(prof_begin(ctx, st, &pp));
  VMLM_TRY(launch_ex(q8_decode_kernel<DecNoGroup>, dim3(static_cast<unsigned>(grid)), dim3(kDecThreads), plan.smem,
                     st, true, plan.c, mw, mp, p, DecNoGroup{0}));
  if (g_profile) VMLM_TRY(prof_end(st, pp, "q8_decode_kernel: " + std::to_string(grid) + " CTAs, clusters of " +
                                                std::to_string(plan.c)));
  return VMLM_OK;
}

// Independent Q8 calls with the same m as one grouped decode launch: a CTA per
// 128-row tile of every call over the tile's whole K, problems ordered by
// descending K so the longest tiles start first. Returns
// VMLM_OK with *done = false when the calls do not fit (the caller then runs
// them one by one).
struct Q8Call {
  const float* a;
  const int8_t* q;
  const float* scale;
  float* c;
  int m, n, k;
};

// A grouped batch of up to 32 tokens with more 128-row tiles than SMs (one
// CTA per tile would run in two waves): q8_decode_sk_kernel, one CTA per SM,
// every CTA streaming an equal share of the batch's k-blocks. The kernel
// makes the digit planes itself for one token, else loads those of one
// q8_planes_group_kernel launch.
// Problems are taken by descending K, as in the one-CTA-per-tile launch.
// *done = false when the batch does not fit (the caller then plans it as
// before).
int run_decode_group_sk(Ctx* ctx, const Q8Call* calls, int count, cudaStream_t st, bool* done) {
  *done = false;
  const int M = calls[0].m;
  if (M < 1 || M > kDecMaxTok) return VMLM_OK;
  int order[kDecMaxGroup];
  for (int i = 0; i < count; ++i) order[i] = i;
  std::stable_sort(order, order + count, [&](int x, int y) { return calls[x].k > calls[y].k; });
  DecGroup grp;
  std::memset(&grp, 0, sizeof(grp));
  grp.count = count;
  long long tiles = 0, total = 0;
  for (int i = 0; i < count; ++i) {
    const Q8Call& q = calls[order[i]];
    DecProblem& pr = grp.prob[i];
    pr.n = q.n;
    pr.k = q.k;
    pr.kb = static_cast<int>(cdiv(q.k, kBlockBytes));
    pr.tile0 = static_cast<int>(tiles);
    pr.kbase = total;
    const long long nt = static_cast<long long>(cdiv(q.n, kTileRows));
    tiles += nt;
    total += nt * pr.kb;
  }
  const int grid = ctx->sms;
  if (tiles <= grid || total < grid) return VMLM_OK;
  const int kbr = static_cast<int>(cdiv(total, grid));
  // The kernel makes the planes itself for one token whose x slice of a share
  // fits one register batch of the plane warps. Otherwise one
  // q8_planes_group_kernel launch makes every problem's planes first: from
  // two tokens on, the in-kernel digit pass delays the first MMA more than
  // the extra launch costs (a 2304-hidden decoder layer's seven linears at
  // m = 2: 25.6 vs 26.8 us).
  const bool planes_mode =
      M > 1 ||
      static_cast<long long>(M) * kbr * (kBlockBytes / 4) > static_cast<long long>(kDecRegChunks) * kDecEpiThreads;
  for (int b = 0; b < grid; ++b) {
    DecSkSegs sg;
    if (!dec_sk_segments(grp.prob, count, total, grid, b, sg)) return VMLM_OK;
  }
  const int rows_b = static_cast<int>(16 * cdiv(3 * M, 16));
  // In planes mode each k-block's planes ride in the ring stage of its W box,
  // so the MMA starts on the first stage (loading the range's planes once, up
  // front, measured 1-2 us slower at m = 2..16 and does not fit at m = 32).
  const int mode = planes_mode ? 1 : 0;
  // three k-blocks per stage (3-D maps) when every problem's rows are whole k-blocks
  int kps = 3;
  for (int i = 0; i < count; ++i)
    if (calls[i].k % 128 != 0) kps = 1;
  int stages = 16;
  while (stages >= 2 && dec_sk_smem_layout(stages, rows_b, kbr, mode, kps).total > static_cast<uint32_t>(kMaxSmem))
    --stages;
  if (stages < 2) return VMLM_OK;
  PlanesGroup pg;
  std::memset(&pg, 0, sizeof(pg));
  char* ws = nullptr;
  if (planes_mode) {
    // every problem's planes [3M][kp] (kp = K rounded up to 16; each region
    // 128-byte aligned), then its exponents and flags [M] each
    size_t bytes = 0;
    for (int i = 0; i < count; ++i)
      bytes += (static_cast<size_t>(3) * M * cdiv(calls[i].k, 16) * 16 + 127) / 128 * 128 + 8ull * M + 128;
    VMLM_TRY(ensure(ctx->grp_planes, bytes));
    ws = static_cast<char*>(ctx->grp_planes.p);
    pg.count = count;
    pg.m = M;
  }
  for (int i = 0; i < count; ++i) {
    const Q8Call& q = calls[order[i]];
    DecProblem& pr = grp.prob[i];
    VMLM_TRY(make_map(&pr.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, q.q, q.k, q.n, q.k, 128, kTileRows));
    if (kps > 1) VMLM_TRY(make_map3(&pr.map3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q.q, q.n, q.k, kTileRows, kps));
    pr.x = q.a;
    pr.w = q.q;
    pr.scale = q.scale;
    pr.out = q.c;
    pr.ldx = q.k;
    pr.ldo = q.n;
    pr.vec_x = (q.k % 4 == 0) && aligned16(q.a);
    if (planes_mode) {
      const int kp = static_cast<int>(cdiv(q.k, 16) * 16);
      int8_t* planes = reinterpret_cast<int8_t*>(ws);
      ws += (static_cast<size_t>(3) * M * kp + 127) / 128 * 128;
      int* exps = reinterpret_cast<int*>(ws);
      ws += (8ull * M + 127) / 128 * 128;
      pr.exps = exps;
      pr.nonfinite = exps + M;
      VMLM_TRY(make_map(&pr.map_p, CU_TENSOR_MAP_DATA_TYPE_UINT8, planes, q.k, 3ull * M, kp, 128,
                        static_cast<uint32_t>(rows_b)));
      pg.prob[i] = PlanesProblem{q.a, planes, exps, exps + M, q.k, kp};
    }
  }
  if (planes_mode)
    VMLM_TRY(launch(q8_planes_group_kernel, dim3(static_cast<unsigned>(M), static_cast<unsigned>(count)),
                    dim3(kPrepThreads), 0, st, true, pg));
  // slots and counters start at zero and are left at zero by every call
  VMLM_TRY(ensure_zeroed(ctx->slots, static_cast<size_t>(tiles) * M * kTileRows * 8, st));
  VMLM_TRY(ensure_zeroed(ctx->counters, static_cast<size_t>(tiles) * 4, st));
  DecSkParams p = {};
  p.m = M;
  p.planes_mode = mode;
  p.rows_b = rows_b;
  p.stages = stages;
  p.kps = kps;
  p.tmem_cols = pow2_at_least(kDecSkMaxSeg * rows_b);
  p.kbr_max = kbr;
  p.grid = grid;
  p.kb_total = total;
  p.slots = static_cast<double*>(ctx->slots.p);
  p.counters = static_cast<int*>(ctx->counters.p);
  p.err = ctx->err;
  p.trace = (g_trace && g_trace_dev == ctx->dev && static_cast<size_t>(grid) <= g_trace_ctas) ? g_trace : nullptr;
  const uint32_t smem = dec_sk_smem_layout(stages, rows_b, kbr, mode, kps).total;
  ProfPair pp;
  if (g_profile) VMLM_TRY(prof_begin(ctx, st, &pp));
  VMLM_TRY(launch(q8_decode_sk_kernel, dim3(static_cast<unsigned>(grid)), dim3(kDecThreads), smem, st, true, p, grp));
  if (g_profile) VMLM_TRY(prof_end(st, pp, "q8_decode_sk_kernel: " + std::to_string(grid) + " CTAs, equal shares"));
  *done = true;
  return VMLM_OK;
}

int run_decode_group(Ctx* ctx, const Q8Call* calls, int count, cudaStream_t st, bool* done) {
  *done = false;
  if (count < 2 || count > kDecMaxGroup) return VMLM_OK;
  const int M = calls[0].m;
  if (M < 1 || M > kDecMaxTok) return VMLM_OK;
  int kb_max = 0, kb_min = 1 << 30;
  for (int i = 0; i < count; ++i) {
    const Q8Call& q = calls[i];
    if (q.m != M || q.n < 1 || q.k < 16 || q.k % 16 || q.k > 131072 || !aligned16(q.q)) return VMLM_OK;
    const int kb = static_cast<int>(cdiv(q.k, kBlockBytes));
    kb_max = std::max(kb_max, kb);
    kb_min = std::min(kb_min, kb);
  }
  VMLM_TRY(run_decode_group_sk(ctx, calls, count, st, done));
  if (*done) return VMLM_OK;
  const int rows_b = static_cast<int>(16 * cdiv(3 * M, 16));
  // When a CTA's x slice over the whole K fits one register batch of the plane
  // warps (the rule plan_decode applies), whole-K CTAs make the planes
  // themselves. Otherwise one q8_planes_group_kernel launch makes every
  // problem's planes first and the kernel loads them (planes mode), on whole-K
  // CTAs where the planes tile fits shared memory, else on the smallest cluster
  // that fits. Splitting K over clusters while the kernel makes the planes in
  // several batches (ten waves of 8-CTA clusters for the C3 set at m = 8)
  // measured slower than the calls one by one.
  const bool planes_mode =
      static_cast<long long>(M) * kb_max * (kBlockBytes / 4) > static_cast<long long>(kDecRegChunks) * kDecEpiThreads;
  int c = 0, kbr = 0, stages = 0;
  for (int cc = 1; cc <= (planes_mode ? kDecMaxCluster : 1) && cc <= kb_min; cc *= 2) {
    const int r = static_cast<int>(cdiv(kb_max, cc));
    int s = r < 16 ? r : 16;
    while (s >= 1 && dec_smem_layout(s, rows_b, r, M, cc).total > static_cast<uint32_t>(kMaxSmem)) --s;
    if (s < 1 || (s < 2 && r > 1)) continue;
    c = cc;
    kbr = r;
    stages = s;
    break;
  }
  if (c == 0) return VMLM_OK;
  int order[kDecMaxGroup];
  for (int i = 0; i < count; ++i) order[i] = i;
  std::stable_sort(order, order + count, [&](int x, int y) { return calls[x].k > calls[y].k; });
  DecGroup grp;
  std::memset(&grp, 0, sizeof(grp));
  grp.count = count;
  PlanesGroup pg;
  std::memset(&pg, 0, sizeof(pg));
  if (planes_mode) {
    // every problem's planes [3M][kp] (kp = K rounded up to 16; each region
    // 128-byte aligned), then its exponents and flags [M] each
    size_t bytes = 0;
    for (int i = 0; i < count; ++i)
      bytes += (static_cast<size_t>(3) * M * cdiv(calls[i].k, 16) * 16 + 127) / 128 * 128 + 8ull * M + 128;
    VMLM_TRY(ensure(ctx->grp_planes, bytes));
    pg.count = count;
    pg.m = M;
  }
  char* ws = static_cast<char*>(ctx->grp_planes.p);
  int tiles = 0;
  for (int i = 0; i < count; ++i) {
    const Q8Call& q = calls[order[i]];
    DecProblem& pr = grp.prob[i];
    VMLM_TRY(make_map(&pr.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, q.q, q.k, q.n, q.k, 128, kTileRows));
    pr.x = q.a;
    pr.w = q.q;
    pr.scale = q.scale;
    pr.out = q.c;
    pr.ldx = q.k;
    pr.ldo = q.n;
    pr.n = q.n;
    pr.k = q.k;
    pr.kb = static_cast<int>(cdiv(q.k, kBlockBytes));
    pr.tile0 = tiles;
    pr.vec_x = (q.k % 4 == 0) && aligned16(q.a);
    tiles += static_cast<int>(cdiv(q.n, kTileRows));
    if (planes_mode) {
      const int kp = static_cast<int>(cdiv(q.k, 16) * 16);
      int8_t* planes = reinterpret_cast<int8_t*>(ws);
      ws += (static_cast<size_t>(3) * M * kp + 127) / 128 * 128;
      int* exps = reinterpret_cast<int*>(ws);
      ws += (8ull * M + 127) / 128 * 128;
      pr.exps = exps;
      pr.nonfinite = exps + M;
      VMLM_TRY(make_map(&pr.map_p, CU_TENSOR_MAP_DATA_TYPE_UINT8, planes, q.k, 3ull * M, kp, 128,
                        static_cast<uint32_t>(rows_b)));
      pg.prob[i] = PlanesProblem{q.a, planes, exps, exps + M, q.k, kp};
    }
  }
  if (planes_mode)
    VMLM_TRY(launch(q8_planes_group_kernel, dim3(static_cast<unsigned>(M), static_cast<unsigned>(count)),
                    dim3(kPrepThreads), 0, st, true, pg));
  DecParams p = {};
  p.m = M;
  p.kps = 1;
  p.cluster = c;
  p.planes_mode = planes_mode ? 1 : 0;
  p.rows_b = rows_b;
  p.kbr_max = kbr;
  p.stages = stages;
  p.tmem_cols = pow2_at_least(rows_b);
  p.err = ctx->err;
  const long long grid = static_cast<long long>(tiles) * c;
  p.trace = (g_trace && g_trace_dev == ctx->dev && static_cast<size_t>(grid) <= g_trace_ctas) ? g_trace : nullptr;
  const uint32_t smem = dec_smem_layout(stages, rows_b, kbr, M, c).total;
  ProfPair pp;
  if (g_profile) VMLM_TRY(prof_begin(ctx, st, &pp));
  // the tensor-map arguments of the ungrouped form are unused here
  VMLM_TRY(launch_ex(q8_decode_kernel<DecGroup>, dim3(static_cast<unsigned>(grid)), dim3(kDecThreads), smem, st,
                     true, c, grp.prob[0].map, grp.prob[0].map, p, grp));
  if (g_profile)
    VMLM_TRY(prof_end(st, pp, "q8_decode_kernel (grouped): " + std::to_string(grid) + " CTAs, clusters of " +
                                  std::to_string(c)));
  *done = true;
  return VMLM_OK;
}

// ------------------------------------------------------ row-sharded calls

// One rank's part of a row-sharded call: its output columns start at col_off
// in every rank's full C (row stride n_total); out[q] / inbox[q] are rank q's
// C and inbox, mapped into this process.
struct Shard {
  int world = 0, rank = 0;
  long long col_off = 0, n_total = 0;
  float* out[kMaxPeers] = {};
  unsigned* inbox[kMaxPeers] = {};
  unsigned* done = nullptr;
  unsigned target = 0;
};

void apply_shard(TcParams& p, const Shard& sh) {
  p.npeers = sh.world;
  p.rank = sh.rank;
  p.col_off = sh.col_off;
  p.ldo = sh.n_total;
  bool vec = (sh.n_total % 4 == 0) && (sh.col_off % 4 == 0);
  for (int q = 0; q < sh.world; ++q) {
    p.peer_out[q] = sh.out[q];
    p.peer_inbox[q] = sh.inbox[q];
    vec = vec && aligned16(sh.out[q]);
  }
  p.vec_out = vec ? 1 : 0;
  p.done_ctr = sh.done;
  p.inbox_target = sh.target;
  p.out = nullptr;
}

// Validate a row-sharded call and fill this rank's part. Rows are split in
// ceil(n / world) blocks; every rank must get at least one.
int shard_check(float* const* c_peers, unsigned* const* inbox_peers, int rank, int world, size_t m, size_t n) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return fail(VMLM_ERR_ARG, "sharded call: rank %d of world %d (1 <= world <= %d)", rank, world, kMaxPeers);
  if (!c_peers || !inbox_peers) return fail(VMLM_ERR_ARG, "sharded call: null peer list");
  for (int q = 0; q < world; ++q)
    if (!c_peers[q] || !inbox_peers[q]) return fail(VMLM_ERR_ARG, "sharded call: null pointer for rank %d", q);
  if (m == 0 || n == 0) return fail(VMLM_ERR_SHAPE, "sharded call: m and n must be positive");
  const size_t rows = (n + world - 1) / world;
  if (rows * (world - 1) >= n) return fail(VMLM_ERR_SHAPE, "sharded call: n=%zu leaves a rank without rows", n);
  return VMLM_OK;
}

int shard_setup(Ctx* ctx, float* const* c_peers, unsigned* const* inbox_peers, int rank, int world, size_t m,
                size_t n, cudaStream_t st, Shard* sh, size_t* nloc) {
  VMLM_TRY(shard_check(c_peers, inbox_peers, rank, world, m, n));
  const size_t rows = (n + world - 1) / world;
  const size_t r0 = rows * rank;
  *nloc = (r0 + rows < n ? r0 + rows : n) - r0;
  VMLM_TRY(ensure_zeroed(ctx->shard_done, 256, st));
  sh->world = world;
  sh->rank = rank;
  sh->col_off = static_cast<long long>(r0);
  sh->n_total = static_cast<long long>(n);
  for (int q = 0; q < world; ++q) {
    sh->out[q] = c_peers[q];
    sh->inbox[q] = inbox_peers[q];
  }
  sh->done = static_cast<unsigned*>(ctx->shard_done.p);
  const unsigned calls = ++g_inbox_calls[reinterpret_cast<uintptr_t>(inbox_peers[rank])];
  sh->target = calls * static_cast<unsigned>(world);
  return VMLM_OK;
}

// ------------------------------------------------------------- Q8 path

// norm_g != nullptr: C = Q8 GEMM of rmsnorm(a) (gain norm_g, norm_eps): the
// norm is fused into the activation encoding, and everything after it reads
// the normalised rows.
// ldo > 0: C rows are ldo elements apart (a column slice of a wider C); else N.
int run_q8(Ctx* c, const float* a, const int8_t* q, const float* scale, float* out, int M, int N, int K,
           cudaStream_t st, const Shard* sh = nullptr, const float* norm_g = nullptr, float norm_eps = 0.f,
           long long ldo = 0) {
  const long long ldc = ldo > 0 ? ldo : N;
  const bool dec_ok = !sh && K > 0 && K % 16 == 0 && K <= 131072 && aligned16(q);
  if (dec_ok && !norm_g) {
    DecPlan dp;
    VMLM_TRY(plan_decode(c, M, N, K, false, &dp));
    if (dp.c > 0) return run_decode(c, a, q, scale, out, M, N, K, st, dp, nullptr, 0, nullptr, nullptr, ldc);
  }
  const int kp = static_cast<int>(cdiv(K, 16) * 16);
  VMLM_TRY(ensure(c->act, static_cast<size_t>(3) * M * (kp ? kp : 16)));
  VMLM_TRY(ensure(c->small, static_cast<size_t>(3) * M * 4 + 64));
  int8_t* planes = static_cast<int8_t*>(c->act.p);
  int* exps = static_cast<int*>(c->small.p);
  int* nonf = exps + M;
  if (norm_g) {
    VMLM_TRY(ensure(c->xn, static_cast<size_t>(M) * (K ? K : 1) * 4));
    float* xn = static_cast<float*>(c->xn.p);
    VMLM_TRY(launch(q8_norm_planes_kernel, dim3(M), dim3(kPrepThreads), 0, st, true, a, static_cast<long long>(K),
                    norm_g, norm_eps, M, K, kp, xn, planes, exps, nonf));
    a = xn;
  } else {
    VMLM_TRY(launch(q8_planes_kernel, dim3(M), dim3(kPrepThreads), 0, st, true, a, static_cast<long long>(K), M, K,
                    kp, planes, exps, nonf));
  }
  if (dec_ok) {
    // x slices too large for the decode kernel's own digit pass: the same
    // kernel on the planes just made (one wave of clusters)
    DecPlan dp;
    VMLM_TRY(plan_decode(c, M, N, K, true, &dp));
    if (dp.c > 0) return run_decode(c, a, q, scale, out, M, N, K, st, dp, planes, kp, exps, nonf, ldc);
  }
  const bool tc_ok = K > 0 && K % 16 == 0 && K <= 131072 && aligned16(q);
  if (!tc_ok) {
    const long long warps = static_cast<long long>(M) * N;
    return launch(q8_generic_kernel, dim3(static_cast<unsigned>(cdiv(warps * 32, 256))), dim3(256), 0, st, true, q,
                  scale, static_cast<const int8_t*>(planes), kp, static_cast<const int*>(exps),
                  static_cast<const int*>(nonf), a, static_cast<long long>(K), out, ldc, M, N,
                  K);
  }
  const int tok = static_cast<int>(cdiv(M < 80 ? M : 80, 16) * 16);
  TcParams p = {};
  p.rows = N;
  p.cols = 3 * M;
  p.bn = 3 * tok;
  p.kb_per_term = static_cast<int>(cdiv(K, 128));
  p.max_terms = 1;
  p.tiles_m = static_cast<int>(cdiv(N, kTileRows));
  p.tiles_n = static_cast<int>(cdiv(M, tok));
  p.tm_fastest = 0;
  p.a_box_elems = 128;
  p.out = out;
  p.ldo = ldc;
  p.vec_out = 0;
  p.scale = scale;
  p.exps = exps;
  p.nonfinite = nonf;
  p.n_tokens = M;
  p.tok_per_tile = tok;
  p.n_out = N;
  p.x = a;
  p.ldx = K;
  p.w = q;
  p.k = K;
  CUtensorMap ma, mb;
  if (sh) apply_shard(p, *sh);
  if (!use_streamk(p, c->sms) && N >= kPairRows) {
    // whole tiles: CTA pairs over 256 weight rows, each SM loading half the planes
    p.tiles_m = static_cast<int>(cdiv(N, kPairRows));
    p.kps = tc2_pick_kps(p.bn, K, kp);
    if (p.kps > 1) {
      VMLM_TRY(make_map3(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, N, K, kTileRows, p.kps));
      VMLM_TRY(make_map3(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, planes, 3ull * M, kp, p.bn / 2, p.kps));
    } else {
      VMLM_TRY(make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, K, N, K, 128, kTileRows));
      VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, planes, K, 3ull * M, kp, 128, p.bn / 2));
    }
    return run_tc2<TcMode::kQ8Swap>(c, st, ma, mb, p, true);
  }
  VMLM_TRY(make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, K, N, K, 128, kTileRows));
  VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, planes, K, 3ull * M, kp, 128, p.bn));
  return run_tc<TcMode::kQ8Swap>(c, st, ma, mb, p, use_streamk(p, c->sms), true);
}

// ------------------------------------------------------------ bf16 path

// bf16 normal mode (more than 80 tokens): split terms written by
// bf16_terms_norm_kernel into buffers of their own, then the tcgen05 GEMM
// with as many term passes as the activations need.
// The tile plan of a bf16 prefill call (tile width, K split, CTA pairs). A
// call split into row chunks runs every chunk with the plan of the whole
// call, so each output is summed in the same order as without chunks.
struct Bf16Plan {
  NormPlan plan;
  bool pairs = false;
  int pair_bn = kPairBn;  // pairs: tile width
  int ksplit = 1;         // pairs: K ranges per tile (2: partials added into a zeroed C)
};

// One-CTA tiles (with a cluster K split where that fills the SMs), or 256-row
// CTA-pair tiles, whole K or K split in two. A pair tile loads fewer operand
// bytes per SM than one-CTA tiles of the same width (B is split between the
// two SMs); split in two, each range adds its partial into C in L2
// (red.global.add; the prep kernel zeroes C first). The cluster K split of
// one-CTA tiles exchanges partials through distributed shared memory, which
// costs several microseconds (remote stores run at about 36 GB/s per SM).
int bf16_norm_plan(Ctx* c, int M, int N, int K, Bf16Plan* out) {
  double t_norm = 0.0;
  VMLM_TRY(plan_norm<TcMode::kBf16Norm>(c, M, N, K, 2, false, &out->plan, &t_norm));
  out->pairs = use_pairs(out->plan, M, N, c->sms);
  out->pair_bn = kPairBn;
  out->ksplit = 1;
  if (out->pairs || M < 2 * kTileRows) return VMLM_OK;
  const double l2_bps = 120e9;   // per SM, as plan_norm
  const double red_bps = 60e9;   // per SM, partial sums added in L2
  const double t_exchange = out->plan.split > 1 ? 3.0e-6 : 0.0;
  double best = t_norm + t_exchange;
  const long long kb = cdiv(K, 64);
  const int pair_slots = c->sms / 2;
  for (int bn : {128, 256}) {
    for (int ks = 1; ks <= 2 && ks <= kb; ++ks) {
      const long long items = cdiv(M, 2 * kTileRows) * cdiv(N, bn) * ks;
      const double waves = static_cast<double>(cdiv(items, pair_slots));
      const double kk = static_cast<double>(kb) / ks;
      const double t_load = kk * (kTileRows + bn / 2) * kBlockBytes / l2_bps;
      const double t_mma = static_cast<double>(kTileRows) * bn * 64 * kk / (11e12 / 2.0);
      const double t_red = ks > 1 ? static_cast<double>(kTileRows) * bn * 4 / red_bps : 0.0;
      const double t = waves * ((t_load > t_mma ? t_load : t_mma) + t_red);
      if (t < best * 0.999) {
        best = t;
        out->pairs = true;
        out->pair_bn = bn;
        out->ksplit = ks;
      }
    }
  }
  return VMLM_OK;
}

int run_bf16_norm(Ctx* c, const float* a, const uint16_t* b, float* out, int M, int N, int K, int kp,
                  cudaStream_t st, const Bf16Plan* force = nullptr) {
  const size_t tbytes = static_cast<size_t>(3) * M * kp * 2;
  if (M != c->norm_m || kp != c->norm_kp) {
    // a new layout: planes and dirty bits start over at zero
    VMLM_TRY(ensure(c->norm_terms, tbytes));
    VMLM_TRY(ensure(c->norm_dirty, static_cast<size_t>(M)));
    VMLM_CUDA(cudaMemsetAsync(c->norm_terms.p, 0, tbytes, st));
    VMLM_CUDA(cudaMemsetAsync(c->norm_dirty.p, 0, static_cast<size_t>(M), st));
    c->norm_m = M;
    c->norm_kp = kp;
  }
  VMLM_TRY(ensure_zeroed(c->norm_flags, 256, st));
  unsigned* fw = static_cast<unsigned*>(c->norm_flags.p);
  unsigned* orword = fw + 32 * c->norm_parity;  // the two words sit on separate 128-byte lines
  unsigned* orword_next = fw + 32 * (c->norm_parity ^ 1u);
  c->norm_parity ^= 1u;
  uint16_t* terms = static_cast<uint16_t*>(c->norm_terms.p);
  Bf16Plan bp;
  if (force)
    bp = *force;
  else
    VMLM_TRY(bf16_norm_plan(c, M, N, K, &bp));
  // a K split of pair tiles adds two partials into C: the prep zeroes it first
  const bool zero_c = bp.pairs && bp.ksplit > 1;
  VMLM_TRY(launch(bf16_terms_norm_kernel, dim3(M), dim3(kNormPrepThreads), 0, st, true, a,
                  static_cast<long long>(K), M, K, kp, static_cast<int>((K % 4 == 0) && aligned16(a)), terms,
                  static_cast<uint8_t*>(c->norm_dirty.p), orword, orword_next, zero_c ? out : nullptr,
                  static_cast<long long>(N), N, static_cast<int>((N % 4 == 0) && aligned16(out))));
  TcParams p = {};
  p.rows = M;
  p.cols = N;
  const NormPlan plan = bp.plan;
  p.bn = plan.bn;
  p.max_terms = 3;
  p.a_box_elems = 64;
  p.kb_per_term = static_cast<int>(cdiv(K, 64));
  p.term_stride = kp;
  p.term_flags = reinterpret_cast<const int*>(orword);
  p.tiles_m = static_cast<int>(cdiv(M, kTileRows));
  p.tiles_n = static_cast<int>(cdiv(N, p.bn));
  p.tm_fastest = 1;
  p.out = out;
  p.ldo = N;
  p.vec_out = (N % 4 == 0) && aligned16(out);
  p.n_tokens = M;
  p.x = a;
  p.ldx = K;
  p.w = b;
  p.k = K;
  CUtensorMap ma, mb;
  VMLM_TRY(make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, terms, 3ull * kp, M, 6ull * kp, 64, kTileRows));
  if (bp.pairs) {
    p.bn = bp.pair_bn;
    p.ksplit = bp.ksplit;
    p.tiles_m = static_cast<int>(cdiv(M, 2 * kTileRows));
    p.tiles_n = static_cast<int>(cdiv(N, p.bn));
    // the terms' rows hold three terms of kp elements: whole k-blocks when kp % 64 == 0
    p.kps = kp % 64 == 0 ? tc2_pick_kps(p.bn, 6ull * kp, 2ull * K) : 1;
    if (p.kps > 1) {
      p.term_kb = kp / 64;
      VMLM_TRY(make_map3(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, terms, M, 6ull * kp, kTileRows, p.kps));
      VMLM_TRY(make_map3(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, N, 2ull * K, p.bn / 2, p.kps));
    } else {
      VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, K, N, 2ull * K, 64, p.bn / 2));
    }
    return run_tc2<TcMode::kBf16Norm>(c, st, ma, mb, p, true);
  }
  VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, K, N, 2ull * K, 64, p.bn));
  return run_tc<TcMode::kBf16Norm>(c, st, ma, mb, p, false, true, plan.split);
}

// ------------------------------------------------------------- f32 path

// C[M,N] (+)= A[M,K] . op(B): nn == false takes B as [N,K] (gemm_nt), nn ==
// true as [K,N] (gemm). Both operands are split into three bf16 terms (B
// transposed to [N][K'] when nn), then the tcgen05 GEMM runs the term pairs
// with i + j <= 2; outputs touching a NaN/Inf row are recomputed exactly.
int run_f32(Ctx* c, const float* a, const float* b, float* out, int M, int N, int K, bool acc, bool nn,
            cudaStream_t st) {
  if (K == 0) {
    // the dot products are empty: C = 0, or C unchanged when accumulating
    if (!acc) VMLM_CUDA(cudaMemsetAsync(out, 0, static_cast<size_t>(M) * N * 4, st));
    return VMLM_OK;
  }
  const int kp = static_cast<int>(cdiv(K, 64) * 64);  // a k-block never runs into the next term
  const size_t ta_bytes = static_cast<size_t>(3) * M * kp * 2, tb_bytes = static_cast<size_t>(3) * N * kp * 2;
  if (M != c->f32_m || N != c->f32_n || kp != c->f32_kp) {
    // a new layout: planes and dirty bits start over at zero
    VMLM_TRY(ensure(c->f32_ta, ta_bytes));
    VMLM_TRY(ensure(c->f32_tb, tb_bytes));
    VMLM_TRY(ensure(c->f32_da, static_cast<size_t>(M)));
    VMLM_TRY(ensure(c->f32_db, static_cast<size_t>(N)));
    VMLM_TRY(ensure(c->f32_nfa, static_cast<size_t>(M) * 4));
    VMLM_TRY(ensure(c->f32_nfb, static_cast<size_t>(N) * 4));
    VMLM_TRY(ensure(c->f32_nft, static_cast<size_t>(N) * 8));
    VMLM_CUDA(cudaMemsetAsync(c->f32_nft.p, 0, static_cast<size_t>(N) * 8, st));
    VMLM_CUDA(cudaMemsetAsync(c->f32_ta.p, 0, ta_bytes, st));
    VMLM_CUDA(cudaMemsetAsync(c->f32_tb.p, 0, tb_bytes, st));
    VMLM_CUDA(cudaMemsetAsync(c->f32_da.p, 0, static_cast<size_t>(M), st));
    VMLM_CUDA(cudaMemsetAsync(c->f32_db.p, 0, static_cast<size_t>(N), st));
    c->f32_m = M;
    c->f32_n = N;
    c->f32_kp = kp;
    c->f32_b_from_t = false;
  }
  VMLM_TRY(ensure_zeroed(c->f32_flags, 512, st));
  unsigned* fw = static_cast<unsigned*>(c->f32_flags.p);  // four words on separate 128-byte lines
  const unsigned par = c->f32_parity;
  c->f32_parity ^= 1u;
  unsigned* or_a = fw + 32 * par;
  unsigned* or_a_next = fw + 32 * (par ^ 1u);
  unsigned* or_b = fw + 64 + 32 * par;
  unsigned* or_b_next = fw + 64 + 32 * (par ^ 1u);
  uint16_t* ta = static_cast<uint16_t*>(c->f32_ta.p);
  uint16_t* tb = static_cast<uint16_t*>(c->f32_tb.p);
  uint8_t* da = static_cast<uint8_t*>(c->f32_da.p);
  uint8_t* db = static_cast<uint8_t*>(c->f32_db.p);
  int* nfa = static_cast<int*>(c->f32_nfa.p);
  int* nfb = static_cast<int*>(c->f32_nfb.p);
  const int vec_a = (K % 4 == 0) && aligned16(a);
  if (nn) {
    // B^T's terms (every plane written, transposed through shared memory) and
    // A's in one launch; B's NaN/Inf column flags alternate between two arrays
    int* nft = static_cast<int*>(c->f32_nft.p);
    nfb = nft + static_cast<size_t>(N) * c->f32_nft_par;
    int* nfb_next = nft + static_cast<size_t>(N) * (c->f32_nft_par ^ 1u);
    c->f32_nft_par ^= 1u;
    const int ntx = static_cast<int>(cdiv(N, kTransTile)), nty = kp / kTransTile;
    VMLM_TRY(launch(f32_terms_nn_kernel, dim3(static_cast<unsigned>(ntx * nty + M)), dim3(kNormPrepThreads), 0, st,
                    true, a, static_cast<long long>(K), M, vec_a, b, static_cast<long long>(N), N, K, kp, ntx, nty,
                    ta, tb, da, nfa, nfb, nfb_next, or_a, or_a_next, or_b, or_b_next));
    c->f32_b_from_t = true;
  } else {
    if (c->f32_b_from_t) {
      // the transposing kernel wrote every plane of B: rewrite them all once
      VMLM_CUDA(cudaMemsetAsync(db, 6, static_cast<size_t>(N), st));
      c->f32_b_from_t = false;
    }
    const int vec_b = (K % 4 == 0) && aligned16(b);
    VMLM_TRY(launch(f32_terms_nt_kernel, dim3(static_cast<unsigned>(M + N)), dim3(kNormPrepThreads), 0, st, true,
                    a, static_cast<long long>(K), M, vec_a, b, static_cast<long long>(K), N, vec_b, K, kp, ta, tb, da,
                    db, nfa, nfb, or_a, or_a_next, or_b, or_b_next));
  }
  NormPlan plan;
  VMLM_TRY(plan_norm<TcMode::kF32Norm>(c, M, N, kp, 2, false, &plan));
  TcParams p = {};
  p.rows = M;
  p.cols = N;
  p.bn = plan.bn;
  p.max_terms = 3;
  p.a_box_elems = 64;
  p.kb_per_term = kp / 64;
  p.term_stride = kp;
  p.term_flags = reinterpret_cast<const int*>(or_a);
  p.term_flags_b = reinterpret_cast<const int*>(or_b);
  p.nf_a = nfa;
  p.nf_b = nfb;
  p.terms_a = ta;
  p.terms_b = tb;
  p.acc_c = acc ? 1 : 0;
  p.tiles_m = static_cast<int>(cdiv(M, kTileRows));
  p.tiles_n = static_cast<int>(cdiv(N, p.bn));
  p.tm_fastest = 1;
  p.out = out;
  p.ldo = N;
  p.vec_out = (N % 4 == 0) && aligned16(out);
  p.k = K;
  CUtensorMap ma, mb;
  VMLM_TRY(make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, ta, 3ull * kp, M, 6ull * kp, 64, kTileRows));
  VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, tb, 3ull * kp, N, 6ull * kp, 64, p.bn));
  return run_tc<TcMode::kF32Norm>(c, st, ma, mb, p, false, true, plan.split);
}

int run_bf16(Ctx* c, const float* a, const uint16_t* b, float* out, int M, int N, int K, cudaStream_t st,
             const Bf16Plan* force = nullptr) {
  const bool tc_ok = K > 0 && K % 8 == 0 && aligned16(b);
  if (!tc_ok) {
    const long long warps = static_cast<long long>(M) * N;
    return launch(bf16_generic_kernel, dim3(static_cast<unsigned>(cdiv(warps * 32, 256))), dim3(256), 0, st, false,
                  b, a, static_cast<long long>(K), out, static_cast<long long>(N), M, N, K);
  }
  const int kp = static_cast<int>(cdiv(K, 8) * 8);
  if (M > 80) return run_bf16_norm(c, a, b, out, M, N, K, kp, st, force);
  VMLM_TRY(ensure(c->act, static_cast<size_t>(3) * M * kp * 2));
  VMLM_TRY(ensure(c->small, static_cast<size_t>(3) * M * 4 + 64));
  uint16_t* terms = static_cast<uint16_t*>(c->act.p);
  int* flags = static_cast<int*>(c->small.p) + 2 * M;
  int* nonf = static_cast<int*>(c->small.p) + M;
  VMLM_TRY(ensure_zeroed(c->sync, 64, st));
  unsigned* done = static_cast<unsigned*>(c->sync.p);
  VMLM_TRY(launch(bf16_terms_kernel, dim3(M), dim3(kPrepThreads), 0, st, true, a, static_cast<long long>(K), M, K,
                  kp, 0, terms, flags, nonf, done));
  TcParams p = {};
  p.max_terms = 1;
  p.a_box_elems = 64;
  p.kb_per_term = static_cast<int>(cdiv(K, 64));
  p.out = out;
  p.ldo = N;
  p.nonfinite = nonf;
  p.term_flags = reinterpret_cast<const int*>(done + 1);
  p.x = a;
  p.ldx = K;
  p.w = b;
  p.k = K;
  CUtensorMap ma, mb;
  {
    const int tok = static_cast<int>(cdiv(M, 16) * 16);
    p.rows = N;
    p.cols = 3 * M;
    p.bn = 3 * tok;
    p.tiles_m = static_cast<int>(cdiv(N, kTileRows));
    p.tiles_n = 1;
    p.tm_fastest = 0;
    p.vec_out = 0;
    p.n_tokens = M;
    p.tok_per_tile = tok;
    p.n_out = N;
    VMLM_TRY(make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, K, N, 2ull * K, 64, kTileRows));
    VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, terms, K, 3ull * M, 2ull * kp, 64, p.bn));
    return run_tc<TcMode::kBf16Swap>(c, st, ma, mb, p, use_streamk(p, c->sms), true);
  }
}

// ---------------------------------------------------------- int8 x int8

// ldo > 0: C rows are ldo elements apart (a column slice of a wider C); else N.
int run_i8i8(Ctx* c, const int8_t* x, const int8_t* w, const float* scale, float* out, int32_t* acc, int M, int N,
             int K, cudaStream_t st, const Shard* sh = nullptr, long long ldo = 0) {
  const bool tc_ok = K > 0 && K % 16 == 0 && aligned16(x) && aligned16(w);
  if (!tc_ok) {
    if (ldo > 0 && ldo != N) return fail(VMLM_ERR_SHAPE, "gemm_i8i8: strided output needs the tensor-core path");
    const long long warps = static_cast<long long>(M) * N;
    return launch(i8i8_generic_kernel, dim3(static_cast<unsigned>(cdiv(warps * 32, 256))), dim3(256), 0, st, false,
                  x, w, scale, out, acc, M, N, K);
  }
  TcParams p = {};
  p.rows = M;
  p.cols = N;
  NormPlan plan;
  VMLM_TRY(plan_norm<TcMode::kI8Norm>(c, M, N, K, 1, true, &plan));
  p.bn = plan.bn;
  p.kb_per_term = static_cast<int>(cdiv(K, 128));
  p.max_terms = 1;
  p.tiles_m = static_cast<int>(cdiv(M, kTileRows));
  p.tiles_n = static_cast<int>(cdiv(N, p.bn));
  p.tm_fastest = 1;
  p.a_box_elems = 128;
  p.out = out;
  p.acc_out = acc;
  p.ldo = ldo > 0 ? ldo : N;
  p.vec_out = (N % 4 == 0) && (p.ldo % 4 == 0) && (!out || aligned16(out)) && (!acc || aligned16(acc));
  p.scale = scale;
  p.n_tokens = M;
  CUtensorMap ma, mb;
  VMLM_TRY(make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, x, K, M, K, 128, kTileRows));
  if (use_pairs(plan, M, N, c->sms)) {
    p.bn = kPairBn;
    p.tiles_m = static_cast<int>(cdiv(M, 2 * kTileRows));
    p.tiles_n = static_cast<int>(cdiv(N, p.bn));
    p.kps = tc2_pick_kps(p.bn, K, K);
    if (p.kps > 1) {
      VMLM_TRY(make_map3(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, x, M, K, kTileRows, p.kps));
      VMLM_TRY(make_map3(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, N, K, kPairBn / 2, p.kps));
    } else {
      VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, K, N, K, 128, kPairBn / 2));
    }
    if (sh) apply_shard(p, *sh);
    return run_tc2<TcMode::kI8Norm>(c, st, ma, mb, p, false);
  }
  VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, K, N, K, 128, p.bn));
  if (sh) apply_shard(p, *sh);
  return run_tc<TcMode::kI8Norm>(c, st, ma, mb, p, false, false, plan.split);
}

// Row-sharded int8 x int8 call whose all-gather is carried by the copy
// engines: the GEMM runs in row chunks on `st`, each chunk written into this
// rank's own C (its column slice); after each chunk, one copy stream per peer
// copies that slice block into the peer's C (2-D copies over NVLink), so the
// transfer of chunk i overlaps the GEMM of chunk i + 1. When a peer stream's
// copies are done it adds 1 to that peer's inbox; this rank's stream then
// waits (bounded) until its own inbox holds every rank's count for the call,
// and for its own outgoing copies. Used when the gather dominates (large
// outputs), where SM stores to peers run below the copy engines' rate.
int run_sharded_ce_i8i8(Ctx* ctx, const int8_t* x, const int8_t* w, const float* scale, const Shard& sh, int M,
                        int nloc, int K, cudaStream_t st) {
  const int world = sh.world, rank = sh.rank;
  float* own = sh.out[rank] + sh.col_off;
  const long long n = sh.n_total;
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    if (!ctx->peer_st[q]) VMLM_CUDA(cudaStreamCreateWithFlags(&ctx->peer_st[q], cudaStreamNonBlocking));
    if (!ctx->peer_done[q]) VMLM_CUDA(cudaEventCreateWithFlags(&ctx->peer_done[q], cudaEventDisableTiming));
  }
  for (cudaEvent_t& e : ctx->chunk_ev)
    if (!e) VMLM_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  // chunks of whole 256-row pair tiles: more of them the more the transfer
  // outweighs the GEMM (it grows with world - 1 against the GEMM's 1 / world)
  const int unit = 2 * kTileRows;
  const int want = std::min(kCeMaxChunks, 2 * world);
  const int chunks = static_cast<int>(std::max(1ll, std::min<long long>(want, M / unit)));
  const int per = static_cast<int>(cdiv(cdiv(M, chunks), unit) * unit);
  for (int r0 = 0, ch = 0; r0 < M; r0 += per, ++ch) {
    const int rows = std::min(per, M - r0);
    VMLM_TRY(run_i8i8(ctx, x + static_cast<long long>(r0) * K, w, scale, own + r0 * n, nullptr, rows, nloc, K, st,
                      nullptr, n));
    VMLM_CUDA(cudaEventRecord(ctx->chunk_ev[ch], st));
    for (int q = 0; q < world; ++q) {
      if (q == rank) continue;
      VMLM_CUDA(cudaStreamWaitEvent(ctx->peer_st[q], ctx->chunk_ev[ch], 0));
      VMLM_CUDA(cudaMemcpy2DAsync(sh.out[q] + sh.col_off + r0 * n, n * 4, own + r0 * n, n * 4,
                                  static_cast<size_t>(nloc) * 4, rows, cudaMemcpyDeviceToDevice, ctx->peer_st[q]));
    }
  }
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    VMLM_TRY(launch(peer_signal_kernel, dim3(1), dim3(32), 0, ctx->peer_st[q], false, sh.inbox[q]));
    VMLM_CUDA(cudaEventRecord(ctx->peer_done[q], ctx->peer_st[q]));
    VMLM_CUDA(cudaStreamWaitEvent(st, ctx->peer_done[q], 0));
  }
  VMLM_TRY(launch(peer_signal_kernel, dim3(1), dim3(32), 0, st, false, sh.inbox[rank]));
  return launch(peer_wait_kernel, dim3(1), dim3(32), 0, st, false, static_cast<const unsigned*>(sh.inbox[rank]),
                sh.target, ctx->err);
}

// Row-sharded calls on more than two GPUs, large outputs: as the copy-engine
// gather, but each finished row chunk is pushed to every peer by
// peer_push_kernel on one stream of its own, beside the GEMM's next chunk (the
// copy engines, one 2-D copy per peer and chunk, reached about 340 GB/s of
// ingress per GPU on eight GPUs), then one count in every peer's inbox and the
// bounded wait for every rank's count. gemm(r0, rows) enqueues the GEMM of
// rows [r0, r0 + rows) into this rank's slice of its own C on st.
template <class F>
int run_sharded_push(Ctx* ctx, const Shard& sh, int M, int nloc, int unit, int chunks, cudaStream_t st, F gemm) {
  const int world = sh.world, rank = sh.rank;
  const float* own = sh.out[rank] + sh.col_off;
  const long long n = sh.n_total;
  if (!ctx->push_st) VMLM_CUDA(cudaStreamCreateWithFlags(&ctx->push_st, cudaStreamNonBlocking));
  if (!ctx->push_done) VMLM_CUDA(cudaEventCreateWithFlags(&ctx->push_done, cudaEventDisableTiming));
  for (cudaEvent_t& e : ctx->chunk_ev)
    if (!e) VMLM_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  PeerDst dst = {};
  for (int q = 0; q < world; ++q) {
    dst.p[q] = sh.out[q] + sh.col_off;
    dst.inbox[q] = sh.inbox[q];
  }
  const int vec = (n % 4 == 0) && (nloc % 4 == 0) && (sh.col_off % 4 == 0) && aligned16(own) ? 1 : 0;
  chunks = static_cast<int>(std::max(1ll, std::min<long long>(std::min(chunks, kCeMaxChunks), M / unit)));
  const int per = static_cast<int>(cdiv(cdiv(M, chunks), unit) * unit);
  for (int r0 = 0, ch = 0; r0 < M; r0 += per, ++ch) {
    const int rows = std::min(per, M - r0);
    VMLM_TRY(gemm(r0, rows));
    VMLM_CUDA(cudaEventRecord(ctx->chunk_ev[ch], st));
    VMLM_CUDA(cudaStreamWaitEvent(ctx->push_st, ctx->chunk_ev[ch], 0));
    PeerDst d = dst;
    for (int q = 0; q < world; ++q) d.p[q] += static_cast<long long>(r0) * n;
    VMLM_TRY(launch(peer_push_kernel, dim3(static_cast<unsigned>(ctx->sms)), dim3(256), 0, ctx->push_st, false,
                    own + static_cast<long long>(r0) * n, n, rows, nloc, d, world, rank, vec));
  }
  VMLM_TRY(launch(peer_signal_all_kernel, dim3(1), dim3(32), 0, ctx->push_st, false, dst, world, rank));
  VMLM_CUDA(cudaEventRecord(ctx->push_done, ctx->push_st));
  VMLM_CUDA(cudaStreamWaitEvent(st, ctx->push_done, 0));
  VMLM_TRY(launch(peer_signal_kernel, dim3(1), dim3(32), 0, st, false, sh.inbox[rank]));
  return launch(peer_wait_kernel, dim3(1), dim3(32), 0, st, false, static_cast<const unsigned*>(sh.inbox[rank]),
                sh.target, ctx->err);
}

// The Q8 form of the copy-engine gather (LM head at many tokens): the whole
// shard's GEMM into this rank's column slice of its own C, then one 2-D copy
// per peer on that peer's copy stream, the peer's count after it, and the
// bounded wait for every rank's count (as run_sharded_ce_i8i8).
int run_sharded_ce_q8(Ctx* ctx, const float* a, const int8_t* q, const float* scale, const Shard& sh, int M, int nloc,
                      int K, cudaStream_t st) {
  const int world = sh.world, rank = sh.rank;
  float* own = sh.out[rank] + sh.col_off;
  const long long n = sh.n_total;
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    if (!ctx->peer_st[p]) VMLM_CUDA(cudaStreamCreateWithFlags(&ctx->peer_st[p], cudaStreamNonBlocking));
    if (!ctx->peer_done[p]) VMLM_CUDA(cudaEventCreateWithFlags(&ctx->peer_done[p], cudaEventDisableTiming));
  }
  if (!ctx->chunk_ev[0]) VMLM_CUDA(cudaEventCreateWithFlags(&ctx->chunk_ev[0], cudaEventDisableTiming));
  VMLM_TRY(run_q8(ctx, a, q, scale, own, M, nloc, K, st, nullptr, nullptr, 0.f, n));
  VMLM_CUDA(cudaEventRecord(ctx->chunk_ev[0], st));
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    VMLM_CUDA(cudaStreamWaitEvent(ctx->peer_st[p], ctx->chunk_ev[0], 0));
    VMLM_CUDA(cudaMemcpy2DAsync(sh.out[p] + sh.col_off, n * 4, own, n * 4, static_cast<size_t>(nloc) * 4, M,
                                cudaMemcpyDeviceToDevice, ctx->peer_st[p]));
    VMLM_TRY(launch(peer_signal_kernel, dim3(1), dim3(32), 0, ctx->peer_st[p], false, sh.inbox[p]));
    VMLM_CUDA(cudaEventRecord(ctx->peer_done[p], ctx->peer_st[p]));
    VMLM_CUDA(cudaStreamWaitEvent(st, ctx->peer_done[p], 0));
  }
  VMLM_TRY(launch(peer_signal_kernel, dim3(1), dim3(32), 0, st, false, sh.inbox[rank]));
  return launch(peer_wait_kernel, dim3(1), dim3(32), 0, st, false, static_cast<const unsigned*>(sh.inbox[rank]),
                sh.target, ctx->err);
}

// ------------------------------------------------------------ host API

// Device address for a host range: registered copy, or a staged upload.
// The device copy of [host, host + bytes) when a registered weight covers it.
bool registered_range(Ctx* c, const void* host, size_t bytes, const void** dptr) {
  auto it = g_reg.upper_bound(reinterpret_cast<uintptr_t>(host));
  if (it == g_reg.begin()) return false;
  --it;
  const uintptr_t h = reinterpret_cast<uintptr_t>(host);
  if (it->second.dev != c->dev || h < it->first || h + bytes > it->first + it->second.bytes) return false;
  *dptr = static_cast<const char*>(it->second.dptr) + (h - it->first);
  return true;
}

int resolve(Ctx* c, const void* host, size_t bytes, DevBuf& stage, cudaStream_t st, const void** dptr) {
  if (registered_range(c, host, bytes, dptr)) return VMLM_OK;
  VMLM_TRY(ensure(stage, bytes));
  VMLM_CUDA(cudaMemcpyAsync(stage.p, host, bytes, cudaMemcpyHostToDevice, st));
  *dptr = stage.p;
  return VMLM_OK;
}

// A host-pointer call over m activation rows, pipelined by chunks of `chunk`
// rows: the copy of chunk i + 1 in (s_in), the compute of chunk i (the
// context's stream) and the copy of chunk i - 1 out (s_out) overlap, and the
// copies in and out use the two directions of the link at once. compute(r0,
// rows) enqueues the work for rows [r0, r0 + rows) on c->stream, reading
// din + r0 * in_row and writing dout + r0 * out_row. Ends as a host call does:
// wait, then read the device error word.
int finish_host_call(Ctx* c, float* host_c, size_t c_bytes, int32_t* host_acc, size_t acc_bytes);

constexpr size_t kPipeChunkRows = 128;  // rows per chunk of a pipelined host call (a multiple)
constexpr size_t kPipeMaxChunks = 8;
std::atomic<int> g_pipe_chunks{4};      // most chunks per pipelined call (vmlm_set_host_pipeline)

template <class F>
int host_pipeline(Ctx* c, size_t m, size_t chunk, const void* host_in, void* din, size_t in_row, void* host_out,
                  void* dout, size_t out_row, F compute) {
  constexpr size_t kEvents = 2 * kPipeMaxChunks + 2;
  if (!c->s_in) {
    VMLM_CUDA(cudaStreamCreateWithFlags(&c->s_in, cudaStreamNonBlocking));
    VMLM_CUDA(cudaStreamCreateWithFlags(&c->s_out, cudaStreamNonBlocking));
    c->pipe_ev.resize(kEvents);
    for (auto& e : c->pipe_ev) VMLM_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  // nothing earlier on the compute stream may still use the staging buffers
  VMLM_CUDA(cudaEventRecord(c->pipe_ev[0], c->stream));
  VMLM_CUDA(cudaStreamWaitEvent(c->s_in, c->pipe_ev[0], 0));
  // every copy in is queued first (events 1 .. nch), so the link is busy
  // while the host is still queueing the GEMMs; events nch + 1 .. mark the
  // chunks' GEMMs for the copies out
  // chunk i covers rows [i * chunk, +chunk); the last one also takes the
  // remainder, so no chunk is shorter than `chunk` rows
  const size_t nch = m / chunk > 0 ? m / chunk : 1;
  if (2 * nch + 2 > kEvents) return fail(VMLM_ERR_SHAPE, "pipelined call: too many chunks");
  auto rows_of = [&](size_t i) { return i + 1 == nch ? m - i * chunk : chunk; };
  for (size_t i = 0; i < nch; ++i) {
    const size_t r0 = i * chunk, rows = rows_of(i);
    VMLM_CUDA(cudaMemcpyAsync(static_cast<char*>(din) + r0 * in_row, static_cast<const char*>(host_in) + r0 * in_row,
                              rows * in_row, cudaMemcpyHostToDevice, c->s_in));
    VMLM_CUDA(cudaEventRecord(c->pipe_ev[1 + i], c->s_in));
  }
  for (size_t i = 0; i < nch; ++i) {
    const size_t r0 = i * chunk, rows = rows_of(i);
    VMLM_CUDA(cudaStreamWaitEvent(c->stream, c->pipe_ev[1 + i], 0));
    VMLM_TRY(compute(r0, rows));
    cudaEvent_t ec = c->pipe_ev[1 + nch + i];
    VMLM_CUDA(cudaEventRecord(ec, c->stream));
    VMLM_CUDA(cudaStreamWaitEvent(c->s_out, ec, 0));
    VMLM_CUDA(cudaMemcpyAsync(static_cast<char*>(host_out) + r0 * out_row, static_cast<char*>(dout) + r0 * out_row,
                              rows * out_row, cudaMemcpyDeviceToHost, c->s_out));
  }
  cudaEvent_t done = c->pipe_ev[1 + 2 * nch];
  VMLM_CUDA(cudaEventRecord(done, c->s_out));
  VMLM_CUDA(cudaStreamWaitEvent(c->stream, done, 0));
  return finish_host_call(c, nullptr, 0, nullptr, 0);
}

// Rows per chunk of a pipelined host call, 0 for a call too small to gain.
size_t pipeline_chunk(size_t m, size_t in_row, size_t out_row, size_t unit = kPipeChunkRows) {
  const size_t most = static_cast<size_t>(g_pipe_chunks.load());
  if (most < 2 || m < 2 * unit || m * (in_row + out_row) < (static_cast<size_t>(2) << 20)) return 0;
  size_t chunk = unit;
  while (m / chunk > most) chunk += unit;
  return chunk;
}

// The status for a non-zero device error word: the VM's OP_EMB messages, or a
// kernel that gave up a bounded wait.
// ------------------------------------------------------- variant kernels

// int4 grouped GEMM: the tiled kernel when every 32-column unit is one
// reference step inside one group and the packed and activation rows are
// 16-byte aligned, else the any-shape kernel. MB = token rows per CTA pass (1, 2, 4 or 8).
template <int MB>
int launch_int4gs(Ctx* c, const float* a, const uint8_t* packed, const float* scale, float* out, int m, int n, int k,
                  int group, int gpr, int order, cudaStream_t st) {
  // a staged token row takes 9 float4 (144 bytes) per 32-column unit
  const int kc_cap = kI4SmemFloats * 4 / (MB * 144) * 32;
  const int kc = k < kc_cap ? k : kc_cap;
  const dim3 grid(static_cast<unsigned>(std::min<long long>(cdiv(n, kI4RowsPerBlock), 8ll * c->sms)),
                  static_cast<unsigned>(cdiv(m, MB)));
  const size_t smem = static_cast<size_t>(MB) * (kc / 32) * 144;
  if (order)
    return launch(int4gs_kernel<MB, 1>, grid, dim3(kI4Warps * 32), smem, st, false, a, packed, scale, out, m, n, k,
                  group, gpr, kc);
  return launch(int4gs_kernel<MB, 0>, grid, dim3(kI4Warps * 32), smem, st, false, a, packed, scale, out, m, n, k, group,
                gpr, kc);
}

int run_int4gs(Ctx* c, const float* a, const uint8_t* packed, const float* scale, float* out, int m, int n, int k,
               int group, int order, cudaStream_t st) {
  if (k == 0) {
    VMLM_CUDA(cudaMemsetAsync(out, 0, static_cast<size_t>(m) * n * 4, st));
    return VMLM_OK;
  }
  const int gpr = static_cast<int>(cdiv(k, group));
  if (m == 1 && k % 32 == 0 && group % 32 == 0 && aligned16(packed) && aligned16(a)) {
    // one token row: the integer (dp4a) form (two rows as two grid rows read the
    // weights twice; the f32 kernel shares them); a chunk of kc columns
    // stages 112 bytes of planes per 32 columns and, for NaN/Inf rows, the floats
    const int kc_cap = kI4SmemFloats * 4 / (112 + 128) * 32;
    const int kc = k < kc_cap ? k : kc_cap;
    const size_t smem = static_cast<size_t>(kc / 32) * (112 + 128);
    // one wave (four CTAs per SM at 60 registers): a CTA stages the row once and
    // streams many row sets
    const dim3 grid(static_cast<unsigned>(std::min<long long>(cdiv(n, kI4RowsPerBlock), 4ll * c->sms)),
                    static_cast<unsigned>(m));
    if (order)
      return launch(int4gs_dp4a_kernel<1>, grid, dim3(kI4Warps * 32), smem, st, false, a, packed, scale, out, n, k,
                    group, gpr, kc);
    return launch(int4gs_dp4a_kernel<0>, grid, dim3(kI4Warps * 32), smem, st, false, a, packed, scale, out, n, k,
                  group, gpr, kc);
  }
  if (k % 32 == 0 && group % 32 == 0 && aligned16(packed) && aligned16(a)) {
    const int mm = m < 8 ? m : 8;
    if (mm == 1) return launch_int4gs<1>(c, a, packed, scale, out, m, n, k, group, gpr, order, st);
    if (mm == 2) return launch_int4gs<2>(c, a, packed, scale, out, m, n, k, group, gpr, order, st);
    if (mm <= 4) return launch_int4gs<4>(c, a, packed, scale, out, m, n, k, group, gpr, order, st);
    return launch_int4gs<8>(c, a, packed, scale, out, m, n, k, group, gpr, order, st);
  }
  const dim3 grid(static_cast<unsigned>(cdiv(static_cast<long long>(m) * n, 8)));
  if (order)
    return launch(int4gs_generic_kernel<1>, grid, dim3(256), 0, st, false, a, packed, scale, out, m, n, k, group, gpr);
  return launch(int4gs_generic_kernel<0>, grid, dim3(256), 0, st, false, a, packed, scale, out, m, n, k, group, gpr);
}

int check_int4(size_t m, size_t n, size_t k, size_t group, int order) {
  VMLM_TRY(check_dims(m, n, k));
  if (group == 0 || group >= (static_cast<size_t>(1) << 31)) return fail(VMLM_ERR_ARG, "int4: group must be >= 1");
  if (order != 0 && order != 1) return fail(VMLM_ERR_ARG, "int4: order must be 0 (packed) or 1 (AVX2 as shipped)");
  if (n * ((k + 1) / 2) >= (static_cast<size_t>(1) << 40)) return fail(VMLM_ERR_SHAPE, "int4: weight too large");
  return VMLM_OK;
}

// int8 + outlier columns: the Q8 GEMM of the int8 body, then the f32 outlier
// terms added in list order.
int run_outlier(Ctx* c, const float* a, const int8_t* q, const float* scale, const float* w, int compact,
                const uint32_t* idx, int n_idx, float* out, int m, int n, int k, cudaStream_t st) {
  VMLM_TRY(run_q8(c, a, q, scale, out, m, n, k, st));
  if (n_idx == 0) return VMLM_OK;
  const dim3 grid(static_cast<unsigned>(cdiv(n, 256)), static_cast<unsigned>(cdiv(m, kOutRows)));
  return launch(outlier_add_kernel, grid, dim3(256), 0, st, true, a, w, compact, idx, n_idx, out, m, n, k, c->err);
}

int device_error(int code) {
  if (code == kDevEmbRange) return fail(VMLM_ERR_OPERATOR, "EMB: row index out of range");
  if (code == kDevEmbFraction) return fail(VMLM_ERR_OPERATOR, "EMB: row index is not an integer");
  if (code == kDevIdxRange) return fail(VMLM_ERR_ARG, "an outlier column index is >= k");
  return fail(VMLM_ERR_DEVICE_TIMEOUT, "a kernel gave up a bounded wait (device code %d)", code);
}

int finish_host_call(Ctx* c, float* host_c, size_t c_bytes, int32_t* host_acc, size_t acc_bytes) {
  if (host_c) VMLM_CUDA(cudaMemcpyAsync(host_c, c->h_c.p, c_bytes, cudaMemcpyDeviceToHost, c->stream));
  if (host_acc) VMLM_CUDA(cudaMemcpyAsync(host_acc, c->h_acc.p, acc_bytes, cudaMemcpyDeviceToHost, c->stream));
  VMLM_CUDA(cudaMemcpyAsync(c->err_host, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  VMLM_CUDA(cudaStreamSynchronize(c->stream));
  if (*c->err_host != 0) {
    const int code = *c->err_host;
    cudaMemset(c->err, 0, sizeof(int));
    if (c->counters.p) cudaMemset(c->counters.p, 0, c->counters.bytes);
    if (c->sync.p) cudaMemset(c->sync.p, 0, c->sync.bytes);
    if (c->slots.p) cudaMemset(c->slots.p, 0, c->slots.bytes);
    if (c->norm_flags.p) cudaMemset(c->norm_flags.p, 0, c->norm_flags.bytes);
    if (c->f32_flags.p) cudaMemset(c->f32_flags.p, 0, c->f32_flags.bytes);
    *c->err_host = 0;
    return device_error(code);
  }
  return VMLM_OK;
}

int host_f32(const float* a, const float* b, float* c, size_t m, size_t n, size_t k, int acc, bool nn,
             const char* what) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(VMLM_ERR_ARG, "%s: null pointer", what);
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const void *da = nullptr, *db = nullptr;
  if (k > 0) {
    VMLM_TRY(resolve(ctx, a, m * k * 4, ctx->h_a, ctx->stream, &da));
    VMLM_TRY(resolve(ctx, b, n * k * 4, ctx->h_b, ctx->stream, &db));
  }
  VMLM_TRY(ensure(ctx->h_c, m * n * 4));
  if (acc) VMLM_CUDA(cudaMemcpyAsync(ctx->h_c.p, c, m * n * 4, cudaMemcpyHostToDevice, ctx->stream));
  VMLM_TRY(run_f32(ctx, static_cast<const float*>(da), static_cast<const float*>(db), static_cast<float*>(ctx->h_c.p),
                   static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), acc != 0, nn, ctx->stream));
  return finish_host_call(ctx, c, m * n * 4, nullptr, 0);
}

int dev_f32(const float* a, const float* b, float* c, size_t m, size_t n, size_t k, int acc, bool nn, void* stream,
            const char* what) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(VMLM_ERR_ARG, "%s: null pointer", what);
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return run_f32(ctx, a, b, c, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), acc != 0, nn, st);
}
// The OP_GEMM arm of Vm::run (core/src/interp.rs:734-812): the VM's guards,
// in its order and with its messages, then the dispatch on B's dtype. The
// guards run before any device work, so a refused call changes nothing.
int op_gemm(unsigned fl, const vmlm_slot* d, const vmlm_slot* a, const vmlm_slot* b, const vmlm_slot* scale,
            bool dev, void* stream) {
  if (!d || !a || !b) return fail(VMLM_ERR_ARG, "op_gemm: null slot");
  const size_t m = a->rows, k = a->cols, b_rows = b->rows, b_cols = b->cols;
  const bool nt = (fl & VMLM_FL_TRANS_B) == 0;
  const bool acc = (fl & VMLM_FL_ACC) != 0;
  auto refuse = [](const char* msg) { return fail(VMLM_ERR_OPERATOR, "%s", msg); };
  // bounds the reference leaves unchecked (it would read or write past a slot)
  auto bounds = [&](size_t n, size_t kb) -> int {
    if (a->dtype != VMLM_DT_F32 || d->dtype != VMLM_DT_F32) return refuse("gemm: activations and output must be f32");
    if (kb != k) return refuse("gemm: K of B differs from cols(A)");
    if (d->rows * d->cols < m * n) return refuse("gemm: output slot smaller than M x N");
    return VMLM_OK;
  };
  if (b->dtype == VMLM_DT_BF16) {
    if (!nt) return refuse("bf16 NN gemm unimplemented");
    if (acc) return refuse("bf16 acc gemm unimplemented");
    VMLM_TRY(bounds(b_rows, b_cols));
    const float* pa = static_cast<const float*>(a->ptr);
    const uint16_t* pb = static_cast<const uint16_t*>(b->ptr);
    float* pc = static_cast<float*>(d->ptr);
    return dev ? vmlm_gemm_nt_bf16_dev(pa, pb, pc, m, b_rows, k, stream) : vmlm_gemm_nt_bf16(pa, pb, pc, m, b_rows, k);
  }
  if (b->dtype == VMLM_DT_I8) {
    if (!nt) return refuse("int8 NN gemm unimplemented");
    if (acc) return refuse("int8 acc gemm unimplemented");
    if (!scale || scale->dtype != VMLM_DT_F32) return refuse("int8 gemm: scale slot must be f32");
    if (scale->rows * scale->cols < b_rows) return refuse("int8 gemm: scale shorter than N rows");
    VMLM_TRY(bounds(b_rows, b_cols));
    const float* pa = static_cast<const float*>(a->ptr);
    const int8_t* pq = static_cast<const int8_t*>(b->ptr);
    const float* ps = static_cast<const float*>(scale->ptr);
    float* pc = static_cast<float*>(d->ptr);
    return dev ? vmlm_gemm_nt_int8_dev(pa, pq, ps, pc, m, b_rows, k, stream)
               : vmlm_gemm_nt_int8(pa, pq, ps, pc, m, b_rows, k);
  }
  if (b->dtype != VMLM_DT_F32) return refuse("gemm operand dtype unsupported");
  const float* pa = static_cast<const float*>(a->ptr);
  const float* pb = static_cast<const float*>(b->ptr);
  float* pc = static_cast<float*>(d->ptr);
  if (nt) {
    VMLM_TRY(bounds(b_rows, b_cols));
    return dev ? vmlm_gemm_nt_f32_dev(pa, pb, pc, m, b_rows, k, acc, stream)
               : vmlm_gemm_nt_f32(pa, pb, pc, m, b_rows, k, acc);
  }
  VMLM_TRY(bounds(b_cols, b_rows));
  return dev ? vmlm_gemm_f32_dev(pa, pb, pc, m, b_cols, k, acc, stream) : vmlm_gemm_f32(pa, pb, pc, m, b_cols, k, acc);
}

}  // namespace

// =================================================================== C ABI

// A .vmb program's constant pool and scratch regions in device memory, with its
// slot table (Vm::load, core/src/interp.rs:123-220) and the OP_LAYERB base.
struct vmlm_pool {
  int dev = -1;
  vmlm::VmbLayout L;
  void* region[4] = {nullptr, nullptr, nullptr, nullptr};  // const, act, state, grad
  uint64_t layer_base = 0;
};

namespace {

void pool_release(vmlm_pool* p) {
  int prev = -1;
  cudaGetDevice(&prev);
  if (p->dev >= 0) cudaSetDevice(p->dev);
  for (void*& r : p->region)
    if (r) {
      cudaFree(r);
      r = nullptr;
    }
  if (prev >= 0) cudaSetDevice(prev);
}

// The device slot i of the pool, with the layer base applied to CONSTANT slots
// and bound-checked as const_ptr_based does (core/src/interp.rs:453-479).
int pool_slot(const vmlm_pool* p, size_t i, vmlm_slot* out, int* kind) {
  if (i >= p->L.slots.size()) return fail(VMLM_ERR_ARG, "pool: slot %zu past the slot table (%zu slots)", i,
                                          p->L.slots.size());
  const vmlm::VmbSlot& s = p->L.slots[i];
  const bool cst = s.kind == vmlm::kVmbSlotConst || s.kind == vmlm::kVmbSlotParam;
  const int r = cst ? 0 : s.kind == vmlm::kVmbSlotState ? 2 : s.kind == vmlm::kVmbSlotGrad ? 3 : 1;
  uint64_t off = s.off;
  if (s.kind == vmlm::kVmbSlotConst && p->layer_base != 0) {
    const uint64_t bytes = static_cast<uint64_t>(s.rows) * s.cols * vmlm::vmb_dtype_size(s.dtype);
    if (off + p->layer_base < off || off + p->layer_base + bytes > p->L.const_len)
      return fail(VMLM_ERR_OPERATOR, "layer base walks past the constant pool: off=%llu base=%llu bytes=%llu limit=%llu",
                  static_cast<unsigned long long>(off), static_cast<unsigned long long>(p->layer_base),
                  static_cast<unsigned long long>(bytes), static_cast<unsigned long long>(p->L.const_len));
    off += p->layer_base;
  }
  if (out) {
    out->ptr = static_cast<char*>(p->region[r]) + off;
    out->rows = s.rows;
    out->cols = s.cols;
    out->dtype = s.dtype;
  }
  if (kind) *kind = static_cast<int>(s.kind);
  return VMLM_OK;
}

}  // namespace

extern "C" {

int vmlm_pool_load(const void* vmb, size_t len, const void* weights, size_t weights_len, vmlm_pool** out) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!out) return fail(VMLM_ERR_ARG, "pool_load: null out");
  *out = nullptr;
  if (!vmb) return fail(VMLM_ERR_ARG, "pool_load: null image");
  vmlm::VmbLayout L;
  const char* msg = "";
  const int rc = vmlm::vmb_parse(static_cast<const uint8_t*>(vmb), len, weights != nullptr, weights_len, &L, &msg);
  if (rc) return fail(rc, "%s", msg);
  std::string audit;
  if (vmlm::vmb_audit(static_cast<const uint8_t*>(vmb), L, &audit)) return fail(VMLM_ERR_OPERATOR, "%s", audit.c_str());
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  vmlm_pool* p = new vmlm_pool();
  p->dev = ctx->dev;
  p->L = std::move(L);
  const uint64_t sizes[4] = {p->L.const_len, p->L.act_bytes, p->L.state_bytes, p->L.grad_bytes};
  for (int r = 0; r < 4; ++r) {
    const size_t bytes = sizes[r] + vmlm::kVmbRegionPad;
    if (cudaMalloc(&p->region[r], bytes) != cudaSuccess) {
      cudaGetLastError();
      pool_release(p);
      delete p;
      return fail(VMLM_ERR_OOM, "pool_load: cudaMalloc of %zu bytes failed", bytes);
    }
    // the VM zeroes its scratch regions (interp.rs:165-187); the pool's slack too
    cudaError_t e = cudaMemset(p->region[r], 0, bytes);
    if (e == cudaSuccess && r == 0 && sizes[0] > 0) {
      const void* src = weights ? weights : static_cast<const char*>(vmb) + p->L.const_off;
      e = cudaMemcpy(p->region[0], src, sizes[0], cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
      pool_release(p);
      delete p;
      return fail(VMLM_ERR_CUDA, "pool_load: %s", cudaGetErrorString(e));
    }
  }
  *out = p;
  return VMLM_OK;
}

int vmlm_pool_free(vmlm_pool* pool) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!pool) return VMLM_OK;
  pool_release(pool);
  delete pool;
  return VMLM_OK;
}

int vmlm_pool_info(const vmlm_pool* pool, size_t* n_const, size_t* n_slots, size_t* region_bytes) {
  if (!pool) return fail(VMLM_ERR_ARG, "pool_info: null pool");
  if (n_const) *n_const = pool->L.consts.size();
  if (n_slots) *n_slots = pool->L.slots.size();
  if (region_bytes) {
    region_bytes[0] = pool->L.const_len;
    region_bytes[1] = pool->L.act_bytes;
    region_bytes[2] = pool->L.state_bytes;
    region_bytes[3] = pool->L.grad_bytes;
  }
  return VMLM_OK;
}

int vmlm_pool_region(const vmlm_pool* pool, int region, void** base) {
  if (!pool || !base) return fail(VMLM_ERR_ARG, "pool_region: null argument");
  if (region < 0 || region > 3) return fail(VMLM_ERR_ARG, "pool_region: region must be 0 (const) .. 3 (grad)");
  *base = pool->region[region];
  return VMLM_OK;
}

int vmlm_pool_slot(const vmlm_pool* pool, size_t slot, vmlm_slot* out, int* kind) {
  if (!pool) return fail(VMLM_ERR_ARG, "pool_slot: null pool");
  return pool_slot(pool, slot, out, kind);
}

int vmlm_pool_layerb(vmlm_pool* pool, float delta) {
  if (!pool) return fail(VMLM_ERR_ARG, "pool_layerb: null pool");
  pool->layer_base = vmlm::vmb_layerb(pool->layer_base, delta);
  return VMLM_OK;
}

int vmlm_pool_layer_base(const vmlm_pool* pool, size_t* base) {
  if (!pool || !base) return fail(VMLM_ERR_ARG, "pool_layer_base: null argument");
  *base = static_cast<size_t>(pool->layer_base);
  return VMLM_OK;
}

int vmlm_pool_find_const(const vmlm_pool* pool, const char* name, size_t* idx) {
  if (!pool || !name || !idx) return fail(VMLM_ERR_ARG, "pool_find_const: null argument");
  const uint32_t h = vmlm::vmb_hash32(name);
  for (size_t i = 0; i < pool->L.consts.size(); ++i)
    if (pool->L.consts[i].hash == h) {
      *idx = i;
      return VMLM_OK;
    }
  return fail(VMLM_ERR_ARG, "const not found");
}

int vmlm_pool_find_slot(const vmlm_pool* pool, const char* name, size_t* idx) {
  if (!pool || !name || !idx) return fail(VMLM_ERR_ARG, "pool_find_slot: null argument");
  const uint32_t h = vmlm::vmb_hash32(name);
  for (size_t i = 0; i < pool->L.slots.size(); ++i)
    if (pool->L.slots[i].name == h) {
      *idx = i;
      return VMLM_OK;
    }
  return fail(VMLM_ERR_ARG, "slot not found");
}

int vmlm_pool_gemm(vmlm_pool* pool, const void* ins, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!pool || !ins) return fail(VMLM_ERR_ARG, "pool_gemm: null argument");
  const uint8_t* b = static_cast<const uint8_t*>(ins);
  if (b[0] != vmlm::kVmbOpGemm) return fail(VMLM_ERR_ARG, "pool_gemm: opcode %u is not OP_GEMM", b[0]);
  uint16_t dt;
  std::memcpy(&dt, b + 2, 2);
  const uint32_t d = vmlm::vmb_u32(b + 4), a = vmlm::vmb_u32(b + 8), bs = vmlm::vmb_u32(b + 12);
  int dev = -1;
  VMLM_CUDA(cudaGetDevice(&dev));
  if (dev != pool->dev) return fail(VMLM_ERR_STATE, "pool_gemm: the pool lives on device %d, current is %d", pool->dev, dev);
  vmlm_slot sd, sa, sb, ss;
  VMLM_TRY(pool_slot(pool, d, &sd, nullptr));
  VMLM_TRY(pool_slot(pool, a, &sa, nullptr));
  VMLM_TRY(pool_slot(pool, bs, &sb, nullptr));
  const bool has_scale = dt < pool->L.slots.size();
  if (has_scale) VMLM_TRY(pool_slot(pool, dt, &ss, nullptr));
  return op_gemm(b[1], &sd, &sa, &sb, has_scale ? &ss : nullptr, true, stream);
}


int vmlm_version(void) { return 100; }

const char* vmlm_last_error(void) { return g_err.c_str(); }

uint64_t vmlm_launch_count(void) { return g_launches.load(); }

int vmlm_init(int device) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (device < 0) {
    int d = 0;
    VMLM_CUDA(cudaGetDevice(&d));
    device = d;
  }
  Ctx* c = nullptr;
  VMLM_TRY(get_ctx(device, &c));
  g_host_dev = device;
  VMLM_CUDA(cudaSetDevice(device));
  return VMLM_OK;
}

int vmlm_unregister_all(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  for (auto& kv : g_reg) {
    cudaSetDevice(kv.second.dev);
    cudaFree(kv.second.dptr);
  }
  g_reg.clear();
  return VMLM_OK;
}

int vmlm_shutdown(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  vmlm_unregister_all();
  for (auto& kv : g_ctx) {
    Ctx* c = kv.second;
    cudaSetDevice(c->dev);
    cudaStreamSynchronize(c->stream);
    for (DevBuf* b : {&c->act, &c->small, &c->slots, &c->counters, &c->shard_done, &c->sync, &c->norm_terms,
                      &c->norm_dirty, &c->norm_flags, &c->f32_ta, &c->f32_tb, &c->f32_da, &c->f32_db, &c->f32_nfa,
                      &c->f32_nfb, &c->f32_nft, &c->f32_flags, &c->h_a, &c->h_c, &c->h_w, &c->h_s, &c->h_acc, &c->h_b, &c->h_g, &c->xn,
                      &c->grp_planes})
      if (b->p) cudaFree(b->p);
    cudaFree(c->err);
    cudaFreeHost(c->err_host);
    for (cudaEvent_t e : c->pipe_ev) cudaEventDestroy(e);
    if (c->s_in) cudaStreamDestroy(c->s_in);
    if (c->s_out) cudaStreamDestroy(c->s_out);
    for (int q = 0; q < kMaxPeers; ++q) {
      if (c->peer_st[q]) cudaStreamDestroy(c->peer_st[q]);
      if (c->peer_done[q]) cudaEventDestroy(c->peer_done[q]);
    }
    for (cudaEvent_t e : c->chunk_ev)
      if (e) cudaEventDestroy(e);
    if (c->push_st) cudaStreamDestroy(c->push_st);
    if (c->push_done) cudaEventDestroy(c->push_done);
    cudaStreamDestroy(c->stream);
    delete c;
  }
  g_ctx.clear();
  g_host_dev = -1;
  return VMLM_OK;
}

int vmlm_register_weight(const void* host_ptr, size_t bytes) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!host_ptr || bytes == 0) return fail(VMLM_ERR_ARG, "register: null pointer or zero size");
  Ctx* c = nullptr;
  VMLM_TRY(host_ctx(&c));
  const uintptr_t h = reinterpret_cast<uintptr_t>(host_ptr);
  auto it = g_reg.lower_bound(h);
  if (it != g_reg.end() && it->first < h + bytes && it->second.dev == c->dev)
    return fail(VMLM_ERR_ARG, "register: range overlaps an existing registration");
  if (it != g_reg.begin()) {
    auto pv = std::prev(it);
    if (pv->first + pv->second.bytes > h && pv->second.dev == c->dev)
      return fail(VMLM_ERR_ARG, "register: range overlaps an existing registration");
  }
  void* d = nullptr;
  VMLM_CUDA(cudaMalloc(&d, bytes));
  cudaError_t e = cudaMemcpy(d, host_ptr, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return fail(VMLM_ERR_CUDA, "register: upload failed: %s", cudaGetErrorString(e));
  }
  g_reg[h] = Reg{bytes, d, c->dev};
  return VMLM_OK;
}

int vmlm_unregister_weight(const void* host_ptr) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_reg.find(reinterpret_cast<uintptr_t>(host_ptr));
  if (it == g_reg.end()) return fail(VMLM_ERR_ARG, "unregister: pointer was not registered");
  cudaSetDevice(it->second.dev);
  cudaFree(it->second.dptr);
  g_reg.erase(it);
  return VMLM_OK;
}

int vmlm_gemm_nt_int8(const float* a, const int8_t* q, const float* scale, float* c, size_t m, size_t n,
                      size_t k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || !scale || (k > 0 && (!a || !q))) return fail(VMLM_ERR_ARG, "gemm_nt_int8: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const void *da = nullptr, *dq = nullptr, *ds = nullptr;
  // large call: A in, the GEMM and C out pipelined by row chunks (the digit
  // planes make every path's sums exact: chunks give the same bits)
  const size_t chunk = k > 0 ? pipeline_chunk(m, k * 4, n * 4) : 0;
  if (chunk) {
    VMLM_TRY(resolve(ctx, q, n * k, ctx->h_w, ctx->stream, &dq));
    VMLM_TRY(resolve(ctx, scale, n * 4, ctx->h_s, ctx->stream, &ds));
    VMLM_TRY(ensure(ctx->h_a, m * k * 4));
    VMLM_TRY(ensure(ctx->h_c, m * n * 4));
    const float* dA = static_cast<const float*>(ctx->h_a.p);
    float* dC = static_cast<float*>(ctx->h_c.p);
    return host_pipeline(ctx, m, chunk, a, ctx->h_a.p, k * 4, c, ctx->h_c.p, n * 4, [&](size_t r0, size_t rows) {
      return run_q8(ctx, dA + r0 * k, static_cast<const int8_t*>(dq), static_cast<const float*>(ds), dC + r0 * n,
                    static_cast<int>(rows), static_cast<int>(n), static_cast<int>(k), ctx->stream);
    });
  }
  VMLM_TRY(resolve(ctx, a, m * k * 4, ctx->h_a, ctx->stream, &da));
  VMLM_TRY(resolve(ctx, q, n * k, ctx->h_w, ctx->stream, &dq));
  VMLM_TRY(resolve(ctx, scale, n * 4, ctx->h_s, ctx->stream, &ds));
  VMLM_TRY(ensure(ctx->h_c, m * n * 4));
  VMLM_TRY(run_q8(ctx, static_cast<const float*>(da), static_cast<const int8_t*>(dq), static_cast<const float*>(ds),
                  static_cast<float*>(ctx->h_c.p), static_cast<int>(m), static_cast<int>(n), static_cast<int>(k),
                  ctx->stream));
  return finish_host_call(ctx, c, m * n * 4, nullptr, 0);
}

int vmlm_gemm_nt_bf16(const float* a, const uint16_t* b, float* c, size_t m, size_t n, size_t k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(VMLM_ERR_ARG, "gemm_nt_bf16: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const void *da = nullptr, *db = nullptr;
  // large prefill call (the tensor-core path with 128-byte-aligned rows): A
  // in, the GEMM and C out pipelined by row chunks, every chunk on the plan
  // of the whole call (the same sums as one call)
  size_t chunk = 0;
  Bf16Plan bp;
  if (k > 0 && k % 8 == 0 && aligned16(b) && m > 80) {
    VMLM_TRY(bf16_norm_plan(ctx, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), &bp));
    chunk = pipeline_chunk(m, k * 4, n * 4, bp.pairs ? 2 * kPipeChunkRows : kPipeChunkRows);
  }
  if (chunk) {
    VMLM_TRY(resolve(ctx, b, n * k * 2, ctx->h_w, ctx->stream, &db));
    VMLM_TRY(ensure(ctx->h_a, m * k * 4));
    VMLM_TRY(ensure(ctx->h_c, m * n * 4));
    const float* dA = static_cast<const float*>(ctx->h_a.p);
    float* dC = static_cast<float*>(ctx->h_c.p);
    return host_pipeline(ctx, m, chunk, a, ctx->h_a.p, k * 4, c, ctx->h_c.p, n * 4, [&](size_t r0, size_t rows) {
      return run_bf16(ctx, dA + r0 * k, static_cast<const uint16_t*>(db), dC + r0 * n, static_cast<int>(rows),
                      static_cast<int>(n), static_cast<int>(k), ctx->stream, &bp);
    });
  }
  VMLM_TRY(resolve(ctx, a, m * k * 4, ctx->h_a, ctx->stream, &da));
  VMLM_TRY(resolve(ctx, b, n * k * 2, ctx->h_w, ctx->stream, &db));
  VMLM_TRY(ensure(ctx->h_c, m * n * 4));
  VMLM_TRY(run_bf16(ctx, static_cast<const float*>(da), static_cast<const uint16_t*>(db),
                    static_cast<float*>(ctx->h_c.p), static_cast<int>(m), static_cast<int>(n), static_cast<int>(k),
                    ctx->stream));
  return finish_host_call(ctx, c, m * n * 4, nullptr, 0);
}

int vmlm_gemm_i8i8(const int8_t* x, const int8_t* w, const float* scale, float* c, int32_t* acc, size_t m, size_t n,
                   size_t k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (k > 131072) return fail(VMLM_ERR_SHAPE, "gemm_i8i8: k > 131072 can overflow the int32 accumulator");
  if (m == 0 || n == 0 || (!c && !acc)) return VMLM_OK;
  if ((c && !scale) || (k > 0 && (!x || !w))) return fail(VMLM_ERR_ARG, "gemm_i8i8: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const void *dx = nullptr, *dw = nullptr, *ds = nullptr;
  // one output of a large call: X in, the GEMM and the output out pipelined
  // by row chunks (integer sums: any tile plan gives the same bits)
  const size_t chunk = (k > 0 && (!c || !acc)) ? pipeline_chunk(m, k, n * 4) : 0;
  if (chunk) {
    VMLM_TRY(resolve(ctx, w, n * k, ctx->h_w, ctx->stream, &dw));
    if (c) VMLM_TRY(resolve(ctx, scale, n * 4, ctx->h_s, ctx->stream, &ds));
    VMLM_TRY(ensure(ctx->h_a, m * k));
    DevBuf& ob = c ? ctx->h_c : ctx->h_acc;
    VMLM_TRY(ensure(ob, m * n * 4));
    const int8_t* dX = static_cast<const int8_t*>(ctx->h_a.p);
    void* host_out = c ? static_cast<void*>(c) : static_cast<void*>(acc);
    return host_pipeline(ctx, m, chunk, x, ctx->h_a.p, k, host_out, ob.p, n * 4, [&](size_t r0, size_t rows) {
      return run_i8i8(ctx, dX + r0 * k, static_cast<const int8_t*>(dw), static_cast<const float*>(ds),
                      c ? static_cast<float*>(ob.p) + r0 * n : nullptr,
                      acc ? static_cast<int32_t*>(ob.p) + r0 * n : nullptr, static_cast<int>(rows),
                      static_cast<int>(n), static_cast<int>(k), ctx->stream);
    });
  }
  VMLM_TRY(resolve(ctx, x, m * k, ctx->h_a, ctx->stream, &dx));
  VMLM_TRY(resolve(ctx, w, n * k, ctx->h_w, ctx->stream, &dw));
  if (c) VMLM_TRY(resolve(ctx, scale, n * 4, ctx->h_s, ctx->stream, &ds));
  if (c) VMLM_TRY(ensure(ctx->h_c, m * n * 4));
  if (acc) VMLM_TRY(ensure(ctx->h_acc, m * n * 4));
  VMLM_TRY(run_i8i8(ctx, static_cast<const int8_t*>(dx), static_cast<const int8_t*>(dw),
                    static_cast<const float*>(ds), c ? static_cast<float*>(ctx->h_c.p) : nullptr,
                    acc ? static_cast<int32_t*>(ctx->h_acc.p) : nullptr, static_cast<int>(m), static_cast<int>(n),
                    static_cast<int>(k), ctx->stream));
  return finish_host_call(ctx, c, m * n * 4, acc, m * n * 4);
}

int vmlm_gemm_nt_f32(const float* a, const float* b, float* c, size_t m, size_t n, size_t k, int acc) {
  return host_f32(a, b, c, m, n, k, acc, false, "gemm_nt_f32");
}

int vmlm_gemm_f32(const float* a, const float* b, float* c, size_t m, size_t n, size_t k, int acc) {
  return host_f32(a, b, c, m, n, k, acc, true, "gemm_f32");
}

int vmlm_gemm_nt_f32_dev(const float* a, const float* b, float* c, size_t m, size_t n, size_t k, int acc,
                         void* stream) {
  return dev_f32(a, b, c, m, n, k, acc, false, stream, "gemm_nt_f32_dev");
}

int vmlm_gemm_f32_dev(const float* a, const float* b, float* c, size_t m, size_t n, size_t k, int acc,
                      void* stream) {
  return dev_f32(a, b, c, m, n, k, acc, true, stream, "gemm_f32_dev");
}

int vmlm_gemm_nt_int8_dev(const float* a, const int8_t* q, const float* scale, float* c, size_t m, size_t n,
                          size_t k, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || !scale || (k > 0 && (!a || !q))) return fail(VMLM_ERR_ARG, "gemm_nt_int8_dev: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return run_q8(ctx, a, q, scale, c, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), st);
}

int vmlm_gemm_nt_bf16_dev(const float* a, const uint16_t* b, float* c, size_t m, size_t n, size_t k,
                          void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(VMLM_ERR_ARG, "gemm_nt_bf16_dev: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return run_bf16(ctx, a, b, c, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), st);
}

int vmlm_gemm_i8i8_dev(const int8_t* x, const int8_t* w, const float* scale, float* c, int32_t* acc, size_t m,
                       size_t n, size_t k, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (k > 131072) return fail(VMLM_ERR_SHAPE, "gemm_i8i8: k > 131072 can overflow the int32 accumulator");
  if (m == 0 || n == 0 || (!c && !acc)) return VMLM_OK;
  if ((c && !scale) || (k > 0 && (!x || !w))) return fail(VMLM_ERR_ARG, "gemm_i8i8_dev: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return run_i8i8(ctx, x, w, scale, c, acc, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), st);
}

int vmlm_rmsnorm_gemm_nt_int8(const float* a, const float* g, float eps, const int8_t* q, const float* scale,
                              float* c, size_t m, size_t n, size_t k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || !scale || (k > 0 && (!a || !q || !g))) return fail(VMLM_ERR_ARG, "rmsnorm_gemm_nt_int8: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const void *da = nullptr, *dq = nullptr, *ds = nullptr, *dg = nullptr;
  VMLM_TRY(resolve(ctx, a, m * k * 4, ctx->h_a, ctx->stream, &da));
  VMLM_TRY(resolve(ctx, q, n * k, ctx->h_w, ctx->stream, &dq));
  VMLM_TRY(resolve(ctx, scale, n * 4, ctx->h_s, ctx->stream, &ds));
  VMLM_TRY(resolve(ctx, g, k * 4, ctx->h_g, ctx->stream, &dg));
  VMLM_TRY(ensure(ctx->h_c, m * n * 4));
  VMLM_TRY(run_q8(ctx, static_cast<const float*>(da), static_cast<const int8_t*>(dq), static_cast<const float*>(ds),
                  static_cast<float*>(ctx->h_c.p), static_cast<int>(m), static_cast<int>(n), static_cast<int>(k),
                  ctx->stream, nullptr, static_cast<const float*>(dg), eps));
  return finish_host_call(ctx, c, m * n * 4, nullptr, 0);
}

int vmlm_rmsnorm_gemm_nt_int8_dev(const float* a, const float* g, float eps, const int8_t* q, const float* scale,
                                  float* c, size_t m, size_t n, size_t k, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || !scale || (k > 0 && (!a || !q || !g))) return fail(VMLM_ERR_ARG, "rmsnorm_gemm_nt_int8_dev: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return run_q8(ctx, a, q, scale, c, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), st, nullptr, g,
                eps);
}

int vmlm_gemv_f32(const float* a, const float* b, float* c, size_t m, size_t k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, 1, k));
  if (m == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(VMLM_ERR_ARG, "gemv_f32: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const void *da = nullptr, *db = nullptr;
  if (k > 0) {
    VMLM_TRY(resolve(ctx, a, m * k * 4, ctx->h_w, ctx->stream, &da));
    VMLM_TRY(resolve(ctx, b, k * 4, ctx->h_a, ctx->stream, &db));
  }
  VMLM_TRY(ensure(ctx->h_c, m * 4));
  VMLM_TRY(vmlm_gemv_f32_dev(static_cast<const float*>(da), static_cast<const float*>(db),
                             static_cast<float*>(ctx->h_c.p), m, k, ctx->stream));
  return finish_host_call(ctx, c, m * 4, nullptr, 0);
}

int vmlm_gemv_f32_dev(const float* a, const float* b, float* c, size_t m, size_t k, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, 1, k));
  if (m == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(VMLM_ERR_ARG, "gemv_f32_dev: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const int vec = (k % 4 == 0) && aligned16(a) && aligned16(b);
  return launch(gemv_f32_kernel, dim3(static_cast<unsigned>(cdiv(static_cast<long long>(m), kGemvWarps))),
                dim3(kGemvWarps * 32), 0, st, false, a, b, c, static_cast<int>(m), static_cast<int>(k), vec);
}

int vmlm_emb(const void* table, int dtype, size_t rows, size_t cols, const float* idx, size_t m, float* out) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (dtype != VMLM_DT_BF16 && dtype != VMLM_DT_F32) return fail(VMLM_ERR_OPERATOR, "EMB: table dtype unsupported");
  if (m == 0 || cols == 0) return VMLM_OK;
  if (!table || !idx || !out) return fail(VMLM_ERR_ARG, "emb: null pointer");
  if (cols >= (static_cast<size_t>(1) << 31)) return fail(VMLM_ERR_SHAPE, "emb: cols must be < 2^31");
  // the VM's checks (core/src/interp.rs:1375-1397), before any device work
  for (size_t t = 0; t < m; ++t) {
    const float r = idx[t];
    if (!(r >= 0.f) || r >= static_cast<float>(rows)) return fail(VMLM_ERR_OPERATOR, "EMB: row index out of range");
    if (static_cast<float>(static_cast<long long>(r)) != r)
      return fail(VMLM_ERR_OPERATOR, "EMB: row index is not an integer");
  }
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const size_t esz = dtype == VMLM_DT_BF16 ? 2 : 4;
  const size_t row_bytes = cols * esz;
  const void* dtab = nullptr;
  std::vector<float> didx(idx, idx + m);
  const uintptr_t h = reinterpret_cast<uintptr_t>(table);
  auto it = g_reg.upper_bound(h);
  bool registered = false;
  if (it != g_reg.begin()) {
    --it;
    if (it->second.dev == ctx->dev && h >= it->first && h + rows * row_bytes <= it->first + it->second.bytes) {
      dtab = static_cast<const char*>(it->second.dptr) + (h - it->first);
      registered = true;
    }
  }
  if (!registered) {
    // only the m rows the call reads go to the device, as rows 0..m-1
    std::vector<char> rowsbuf(m * row_bytes);
    for (size_t t = 0; t < m; ++t) {
      std::memcpy(rowsbuf.data() + t * row_bytes,
                  static_cast<const char*>(table) + static_cast<size_t>(idx[t]) * row_bytes, row_bytes);
      didx[t] = static_cast<float>(t);
    }
    VMLM_TRY(ensure(ctx->h_w, rowsbuf.size()));
    VMLM_CUDA(cudaMemcpyAsync(ctx->h_w.p, rowsbuf.data(), rowsbuf.size(), cudaMemcpyHostToDevice, ctx->stream));
    VMLM_CUDA(cudaStreamSynchronize(ctx->stream));  // rowsbuf is pageable and goes out of scope
    dtab = ctx->h_w.p;
  }
  VMLM_TRY(ensure(ctx->h_a, m * 4));
  VMLM_CUDA(cudaMemcpyAsync(ctx->h_a.p, didx.data(), m * 4, cudaMemcpyHostToDevice, ctx->stream));
  VMLM_TRY(ensure(ctx->h_c, m * cols * 4));
  VMLM_TRY(launch(emb_kernel, dim3(static_cast<unsigned>(m), static_cast<unsigned>(cdiv(cols, 1024))), dim3(256), 0,
                  ctx->stream, false, dtab, dtype, static_cast<long long>(registered ? rows : m),
                  static_cast<int>(cols), static_cast<const float*>(ctx->h_a.p), static_cast<int>(m),
                  static_cast<float*>(ctx->h_c.p), ctx->err));
  VMLM_CUDA(cudaStreamSynchronize(ctx->stream));  // didx is pageable
  return finish_host_call(ctx, out, m * cols * 4, nullptr, 0);
}

int vmlm_emb_dev(const void* table, int dtype, size_t rows, size_t cols, const float* idx, size_t m, float* out,
                 void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (dtype != VMLM_DT_BF16 && dtype != VMLM_DT_F32) return fail(VMLM_ERR_OPERATOR, "EMB: table dtype unsupported");
  if (m == 0 || cols == 0) return VMLM_OK;
  if (!table || !idx || !out) return fail(VMLM_ERR_ARG, "emb_dev: null pointer");
  if (cols >= (static_cast<size_t>(1) << 31) || m >= (static_cast<size_t>(1) << 31))
    return fail(VMLM_ERR_SHAPE, "emb_dev: m and cols must be < 2^31");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return launch(emb_kernel, dim3(static_cast<unsigned>(m), static_cast<unsigned>(cdiv(cols, 1024))), dim3(256), 0, st,
                false, table, dtype, static_cast<long long>(rows), static_cast<int>(cols), idx, static_cast<int>(m),
                out, ctx->err);
}

int vmlm_gemm_nt_int8_batch_dev(const vmlm_q8_call* calls, size_t count, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (count == 0) return VMLM_OK;
  if (!calls) return fail(VMLM_ERR_ARG, "gemm_nt_int8_batch_dev: null call list");
  for (size_t i = 0; i < count; ++i) {
    const vmlm_q8_call& q = calls[i];
    VMLM_TRY(check_dims(q.m, q.n, q.k));
    if (q.m > 0 && q.n > 0 && (!q.c || !q.scale || (q.k > 0 && (!q.a || !q.q))))
      return fail(VMLM_ERR_ARG, "gemm_nt_int8_batch_dev: null pointer in call %zu", i);
  }
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  std::vector<Q8Call> qc;
  for (size_t i = 0; i < count; ++i)
    if (calls[i].m > 0 && calls[i].n > 0)
      qc.push_back(Q8Call{calls[i].a, calls[i].q, calls[i].scale, calls[i].c, static_cast<int>(calls[i].m),
                          static_cast<int>(calls[i].n), static_cast<int>(calls[i].k)});
  for (size_t i0 = 0; i0 < qc.size(); i0 += kDecMaxGroup) {
    const int cnt = static_cast<int>(std::min<size_t>(kDecMaxGroup, qc.size() - i0));
    bool done = false;
    VMLM_TRY(run_decode_group(ctx, qc.data() + i0, cnt, st, &done));
    if (done) continue;
    for (int i = 0; i < cnt; ++i) {
      const Q8Call& q = qc[i0 + i];
      VMLM_TRY(run_q8(ctx, q.a, q.q, q.scale, q.c, q.m, q.n, q.k, st));
    }
  }
  return VMLM_OK;
}

int vmlm_gemm_nt_int4_gs(const float* a, const uint8_t* packed, const float* scale, float* c, size_t m, size_t n,
                         size_t k, size_t group, int order) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_int4(m, n, k, group, order));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !packed || !scale))) return fail(VMLM_ERR_ARG, "gemm_nt_int4_gs: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const void *da = nullptr, *dp = nullptr, *ds = nullptr;
  if (k > 0) {
    VMLM_TRY(resolve(ctx, a, m * k * 4, ctx->h_a, ctx->stream, &da));
    VMLM_TRY(resolve(ctx, packed, n * ((k + 1) / 2), ctx->h_w, ctx->stream, &dp));
    VMLM_TRY(resolve(ctx, scale, n * ((k + group - 1) / group) * 4, ctx->h_s, ctx->stream, &ds));
  }
  VMLM_TRY(ensure(ctx->h_c, m * n * 4));
  VMLM_TRY(run_int4gs(ctx, static_cast<const float*>(da), static_cast<const uint8_t*>(dp),
                      static_cast<const float*>(ds), static_cast<float*>(ctx->h_c.p), static_cast<int>(m),
                      static_cast<int>(n), static_cast<int>(k), static_cast<int>(group), order, ctx->stream));
  return finish_host_call(ctx, c, m * n * 4, nullptr, 0);
}

int vmlm_gemm_nt_int4_gs_dev(const float* a, const uint8_t* packed, const float* scale, float* c, size_t m, size_t n,
                             size_t k, size_t group, int order, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_int4(m, n, k, group, order));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !packed || !scale))) return fail(VMLM_ERR_ARG, "gemm_nt_int4_gs_dev: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return run_int4gs(ctx, a, packed, scale, c, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k),
                    static_cast<int>(group), order, st);
}

int vmlm_gemm_nt_int8_outlier(const float* a, const int8_t* q, const float* scale, const float* w,
                              const uint32_t* idx, size_t n_idx, float* c, size_t m, size_t n, size_t k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (n_idx > k) return fail(VMLM_ERR_ARG, "gemm_nt_int8_outlier: more outlier columns than k");
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !q || !scale)) || (n_idx > 0 && (!w || !idx)))
    return fail(VMLM_ERR_ARG, "gemm_nt_int8_outlier: null pointer");
  for (size_t t = 0; t < n_idx; ++t)
    if (idx[t] >= k) return fail(VMLM_ERR_ARG, "gemm_nt_int8_outlier: outlier column index %u >= k", idx[t]);
  Ctx* ctx = nullptr;
  VMLM_TRY(host_ctx(&ctx));
  const void *da = nullptr, *dq = nullptr, *ds = nullptr, *dw = nullptr, *di = nullptr;
  int compact = 0;
  if (k > 0) {
    VMLM_TRY(resolve(ctx, a, m * k * 4, ctx->h_a, ctx->stream, &da));
    VMLM_TRY(resolve(ctx, q, n * k, ctx->h_w, ctx->stream, &dq));
    VMLM_TRY(resolve(ctx, scale, n * 4, ctx->h_s, ctx->stream, &ds));
  }
  std::vector<float> cols;
  if (n_idx > 0) {
    VMLM_TRY(resolve(ctx, idx, n_idx * 4, ctx->h_g, ctx->stream, &di));
    if (!registered_range(ctx, w, n * k * 4, &dw)) {
      // only the outlier columns the call reads go to the device, as [n][n_idx]
      cols.resize(n * n_idx);
      for (size_t j = 0; j < n; ++j)
        for (size_t t = 0; t < n_idx; ++t) cols[j * n_idx + t] = w[j * k + idx[t]];
      VMLM_TRY(ensure(ctx->h_b, cols.size() * 4));
      VMLM_CUDA(cudaMemcpyAsync(ctx->h_b.p, cols.data(), cols.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
      dw = ctx->h_b.p;
      compact = 1;
    }
  }
  VMLM_TRY(ensure(ctx->h_c, m * n * 4));
  VMLM_TRY(run_outlier(ctx, static_cast<const float*>(da), static_cast<const int8_t*>(dq),
                       static_cast<const float*>(ds), static_cast<const float*>(dw), compact,
                       static_cast<const uint32_t*>(di), static_cast<int>(n_idx), static_cast<float*>(ctx->h_c.p),
                       static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), ctx->stream));
  if (!cols.empty()) VMLM_CUDA(cudaStreamSynchronize(ctx->stream));  // cols is pageable
  return finish_host_call(ctx, c, m * n * 4, nullptr, 0);
}

int vmlm_gemm_nt_int8_outlier_dev(const float* a, const int8_t* q, const float* scale, const float* w, int compact,
                                  const uint32_t* idx, size_t n_idx, float* c, size_t m, size_t n, size_t k,
                                  void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (n_idx > k) return fail(VMLM_ERR_ARG, "gemm_nt_int8_outlier_dev: more outlier columns than k");
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || (k > 0 && (!a || !q || !scale)) || (n_idx > 0 && (!w || !idx)))
    return fail(VMLM_ERR_ARG, "gemm_nt_int8_outlier_dev: null pointer");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return run_outlier(ctx, a, q, scale, w, compact ? 1 : 0, idx, static_cast<int>(n_idx), c, static_cast<int>(m),
                     static_cast<int>(n), static_cast<int>(k), st);
}

int vmlm_gather_columns_dev(const float* w, const uint32_t* idx, size_t n_idx, size_t n, size_t k, float* wo,
                            void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(n_idx, n, k));
  if (n_idx == 0 || n == 0) return VMLM_OK;
  if (!w || !idx || !wo) return fail(VMLM_ERR_ARG, "gather_columns_dev: null pointer");
  if (n * n_idx >= (static_cast<size_t>(1) << 40)) return fail(VMLM_ERR_SHAPE, "gather_columns_dev: too large");
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return launch(gather_columns_kernel, dim3(static_cast<unsigned>(cdiv(static_cast<long long>(n * n_idx), 256))),
                dim3(256), 0, st, false, w, idx, static_cast<int>(n_idx), wo, static_cast<int>(n),
                static_cast<int>(k), ctx->err);
}

int vmlm_op_gemm(unsigned fl, const vmlm_slot* d, const vmlm_slot* a, const vmlm_slot* b, const vmlm_slot* scale) {
  return op_gemm(fl, d, a, b, scale, false, nullptr);
}

int vmlm_op_gemm_dev(unsigned fl, const vmlm_slot* d, const vmlm_slot* a, const vmlm_slot* b, const vmlm_slot* scale,
                     void* stream) {
  return op_gemm(fl, d, a, b, scale, true, stream);
}

int vmlm_trace_enable(int max_ctas) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (g_trace) {
    cudaSetDevice(g_trace_dev);
    cudaFree(g_trace);
    g_trace = nullptr;
    g_trace_ctas = 0;
  }
  if (max_ctas <= 0) return VMLM_OK;
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  const size_t bytes = static_cast<size_t>(max_ctas) * kTraceSlots * sizeof(unsigned long long);
  VMLM_CUDA(cudaMalloc(&g_trace, bytes));
  VMLM_CUDA(cudaMemset(g_trace, 0, bytes));
  g_trace_ctas = static_cast<size_t>(max_ctas);
  g_trace_dev = ctx->dev;
  return VMLM_OK;
}

int vmlm_trace_take(uint64_t* host, size_t n_values) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!g_trace) return fail(VMLM_ERR_STATE, "trace: not enabled");
  const size_t have = g_trace_ctas * kTraceSlots;
  if (!host || n_values > have) return fail(VMLM_ERR_ARG, "trace: buffer larger than the trace");
  VMLM_CUDA(cudaDeviceSynchronize());
  VMLM_CUDA(cudaMemcpy(host, g_trace, n_values * sizeof(uint64_t), cudaMemcpyDeviceToHost));
  return VMLM_OK;
}

int vmlm_profile_enable(int on) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  g_profile = on != 0;
  return VMLM_OK;
}

int vmlm_profile_kernel(char* buf, size_t n) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!buf || n == 0) return fail(VMLM_ERR_ARG, "vmlm_profile_kernel: null buffer");
  snprintf(buf, n, "%s", g_prof_last.c_str());
  return VMLM_OK;
}

int vmlm_profile_take(double* gemm_ms, uint64_t* launches) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  double total = 0.0;
  uint64_t n = 0;
  for (ProfPair& pp : g_prof_live) {
    VMLM_CUDA(cudaEventSynchronize(pp.b));
    float ms = 0.f;
    VMLM_CUDA(cudaEventElapsedTime(&ms, pp.a, pp.b));
    total += ms;
    ++n;
    g_prof_free.push_back(pp);
  }
  g_prof_live.clear();
  if (gemm_ms) *gemm_ms = total;
  if (launches) *launches = n;
  return VMLM_OK;
}

// ------------------------------------------------------------ row-sharded

int vmlm_ipc_handle(const void* dptr, void* handle) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!dptr || !handle) return fail(VMLM_ERR_ARG, "ipc_handle: null pointer");
  typedef CUresult (*RangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range = nullptr;
  if (!range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    VMLM_CUDA(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !fn) return fail(VMLM_ERR_CUDA, "cuMemGetAddressRange not available");
    range = reinterpret_cast<RangeFn>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dptr)) != CUDA_SUCCESS)
    return fail(VMLM_ERR_ARG, "ipc_handle: %p is not device memory", dptr);
  cudaIpcMemHandle_t h;
  VMLM_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  const uint64_t off = reinterpret_cast<uint64_t>(dptr) - static_cast<uint64_t>(base);
  std::memcpy(handle, &h, sizeof h);
  std::memcpy(static_cast<char*>(handle) + sizeof h, &off, sizeof off);
  return VMLM_OK;
}

int vmlm_ipc_open(const void* handle, void** dptr) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!handle || !dptr) return fail(VMLM_ERR_ARG, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  uint64_t off = 0;
  std::memcpy(&h, handle, sizeof h);
  std::memcpy(&off, static_cast<const char*>(handle) + sizeof h, sizeof off);
  const std::string key(reinterpret_cast<const char*>(&h), sizeof h);
  auto it = g_ipc.find(key);
  if (it == g_ipc.end()) {
    void* base = nullptr;
    VMLM_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    it = g_ipc.emplace(key, IpcMap{base, 0}).first;
  }
  ++it->second.refs;
  *dptr = static_cast<char*>(it->second.base) + off;
  g_ipc_users[reinterpret_cast<uintptr_t>(*dptr)] = key;
  return VMLM_OK;
}

int vmlm_ipc_close(void* dptr) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto u = g_ipc_users.find(reinterpret_cast<uintptr_t>(dptr));
  if (u == g_ipc_users.end()) return fail(VMLM_ERR_ARG, "ipc_close: %p was not opened by vmlm_ipc_open", dptr);
  auto it = g_ipc.find(u->second);
  g_ipc_users.erase(u);
  if (it != g_ipc.end() && --it->second.refs == 0) {
    const cudaError_t e = cudaIpcCloseMemHandle(it->second.base);
    g_ipc.erase(it);
    if (e != cudaSuccess) return fail(VMLM_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  }
  return VMLM_OK;
}

int vmlm_sharded_reset(unsigned* inbox) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!inbox) return fail(VMLM_ERR_ARG, "sharded_reset: null pointer");
  VMLM_CUDA(cudaMemset(inbox, 0, sizeof(unsigned)));
  g_inbox_calls.erase(reinterpret_cast<uintptr_t>(inbox));
  return VMLM_OK;
}

int vmlm_sharded_gemm_nt_int8_dev(const float* a, const int8_t* q_shard, const float* scale_shard,
                                  float* const* c_peers, unsigned* const* inbox_peers, int rank, int world, size_t m,
                                  size_t n, size_t k, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (!a || !q_shard || !scale_shard) return fail(VMLM_ERR_ARG, "sharded_gemm_nt_int8_dev: null pointer");
  if (k == 0 || k % 16 != 0 || k > 131072 || !aligned16(q_shard))
    return fail(VMLM_ERR_SHAPE, "sharded_gemm_nt_int8_dev: needs k %% 16 == 0, k <= 131072, 16-byte aligned q");
  VMLM_TRY(shard_check(c_peers, inbox_peers, rank, world, m, n));
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  Shard sh;
  size_t nloc = 0;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  VMLM_TRY(shard_setup(ctx, c_peers, inbox_peers, rank, world, m, n, st, &sh, &nloc));
  const double peer_bytes = 4.0 * m * nloc * (world - 1);
  // Large outputs on two GPUs: the copy engines carry the gather after the
  // GEMM. On more GPUs the fused epilogue stores, which overlap the GEMM, are
  // faster (C4 at 64 tokens on eight GPUs: 116 µs fused, 126 pushed after the
  // GEMM, 150 by the copy engines; GEMM + NCCL all-gather 109).
  if (world == 2 && peer_bytes >= kCeMinPeerBytes)
    return run_sharded_ce_q8(ctx, a, q_shard, scale_shard, sh, static_cast<int>(m), static_cast<int>(nloc),
                             static_cast<int>(k), st);
  return run_q8(ctx, a, q_shard, scale_shard, nullptr, static_cast<int>(m), static_cast<int>(nloc),
                static_cast<int>(k), st, &sh);
}

int vmlm_sharded_gemm_i8i8_dev(const int8_t* x, const int8_t* w_shard, const float* scale_shard,
                               float* const* c_peers, unsigned* const* inbox_peers, int rank, int world, size_t m,
                               size_t n, size_t k, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (!x || !w_shard || !scale_shard) return fail(VMLM_ERR_ARG, "sharded_gemm_i8i8_dev: null pointer");
  if (k == 0 || k % 16 != 0 || k > 131072 || !aligned16(x) || !aligned16(w_shard))
    return fail(VMLM_ERR_SHAPE, "sharded_gemm_i8i8_dev: needs k %% 16 == 0, k <= 131072, 16-byte aligned x and w");
  VMLM_TRY(shard_check(c_peers, inbox_peers, rank, world, m, n));
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  Shard sh;
  size_t nloc = 0;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  VMLM_TRY(shard_setup(ctx, c_peers, inbox_peers, rank, world, m, n, st, &sh, &nloc));
  // large outputs: the copy engines carry the gather, the GEMM in row chunks overlapping it
  const double peer_bytes = 4.0 * m * nloc * (world - 1);
  // More than two GPUs: each row chunk pushed by peer_push_kernel beside the
  // next chunk's GEMM (C5 on eight GPUs: 754 µs, against 1242 by the copy
  // engines, 925 by fused epilogue stores and 791 for GEMM + NCCL all-gather).
  if (world > 2 && peer_bytes >= kCeMinPeerBytes && m >= 512) {
    float* own = sh.out[sh.rank] + sh.col_off;
    return run_sharded_push(ctx, sh, static_cast<int>(m), static_cast<int>(nloc), 2 * kTileRows, 2 * world, st,
                            [&](int r0, int rows) {
                              return run_i8i8(ctx, x + static_cast<long long>(r0) * k, w_shard, scale_shard,
                                              own + static_cast<long long>(r0) * n, nullptr, rows,
                                              static_cast<int>(nloc), static_cast<int>(k), st, nullptr, n);
                            });
  }
  if (world > 1 && peer_bytes >= kCeMinPeerBytes && m >= 512)
    return run_sharded_ce_i8i8(ctx, x, w_shard, scale_shard, sh, static_cast<int>(m), static_cast<int>(nloc),
                               static_cast<int>(k), st);
  return run_i8i8(ctx, x, w_shard, scale_shard, nullptr, nullptr, static_cast<int>(m), static_cast<int>(nloc),
                  static_cast<int>(k), st, &sh);
}

int vmlm_probe_mma_peak(int kind, int iters, double* tops, double* ms) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (kind != 0 && kind != 1) return fail(VMLM_ERR_ARG, "probe_mma_peak: kind must be 0 (bf16) or 1 (int8)");
  if (iters < 1 || iters > kProbeMaxIters)
    return fail(VMLM_ERR_ARG, "probe_mma_peak: iters must be in [1, %d]", kProbeMaxIters);
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  auto kern = kind == 0 ? mma_peak_kernel<0> : mma_peak_kernel<1>;
  VMLM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem));
  cudaEvent_t e0, e1;
  VMLM_CUDA(cudaEventCreate(&e0));
  VMLM_CUDA(cudaEventCreate(&e1));
  cudaEventRecord(e0, ctx->stream);
  const int rc = launch(kern, dim3(static_cast<unsigned>(ctx->sms)), dim3(kProbeThreads), kProbeSmem, ctx->stream,
                        false, iters, ctx->err);
  cudaEventRecord(e1, ctx->stream);
  const cudaError_t se = cudaEventSynchronize(e1);
  float t = 0.f;
  cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  VMLM_TRY(rc);
  if (se != cudaSuccess) return fail(VMLM_ERR_CUDA, "probe_mma_peak: %s", cudaGetErrorString(se));
  VMLM_TRY(vmlm_sync(nullptr));
  const double ops = static_cast<double>(ctx->sms) * iters * 4.0 * 2.0 * 128.0 * 256.0 * (kind == 0 ? 16.0 : 32.0);
  if (ms) *ms = t;
  if (tops) *tops = t > 0.f ? ops / (t * 1e-3) / 1e12 : 0.0;
  return VMLM_OK;
}

int vmlm_set_host_pipeline(int max_chunks) {
  if (max_chunks < 0 || max_chunks > static_cast<int>(kPipeMaxChunks))
    return fail(VMLM_ERR_ARG, "set_host_pipeline: max_chunks must be in [0, %d]", static_cast<int>(kPipeMaxChunks));
  g_pipe_chunks.store(max_chunks == 0 ? 4 : max_chunks);
  return VMLM_OK;
}

int vmlm_sync(void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  int dev = -1;
  VMLM_CUDA(cudaGetDevice(&dev));
  // The allocation-free entry point keeps its own error word; read it first.
  // A device that has only seen allocation-free calls gets no context here,
  // so this call allocates nothing for such a caller either.
  int na_code = 0;
  VMLM_TRY(na_take_error(dev, &na_code));
  if (na_code != 0 && g_ctx.find(dev) == g_ctx.end()) return device_error(na_code);
  if (na_ready(dev) && g_ctx.find(dev) == g_ctx.end()) {
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : cudaStreamLegacy;
    VMLM_CUDA(cudaStreamSynchronize(st));
    return VMLM_OK;
  }
  Ctx* ctx = nullptr;
  VMLM_TRY(current_ctx(&ctx));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  VMLM_CUDA(cudaStreamSynchronize(st));
  if (na_code != 0) return device_error(na_code);
  int code = 0;
  VMLM_CUDA(cudaMemcpy(&code, ctx->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    // clear on the same stream and wait, so the next call on any stream sees zeros
    cudaMemsetAsync(ctx->err, 0, sizeof(int), st);
    if (ctx->counters.p) cudaMemsetAsync(ctx->counters.p, 0, ctx->counters.bytes, st);
    if (ctx->sync.p) cudaMemsetAsync(ctx->sync.p, 0, ctx->sync.bytes, st);
    if (ctx->slots.p) cudaMemsetAsync(ctx->slots.p, 0, ctx->slots.bytes, st);
    if (ctx->shard_done.p) cudaMemsetAsync(ctx->shard_done.p, 0, ctx->shard_done.bytes, st);
    VMLM_CUDA(cudaStreamSynchronize(st));
    return device_error(code);
  }
  return VMLM_OK;
}

}  // extern "C"

// ====================================================== allocation-free Q8
//
// vmlm_gemm_nt_int8_dev_noalloc runs the Q8 path with every byte of scratch
// (activation digit planes, per-token exponents and flags, split-tile slots
// and counters, the device error word) taken from one fixed array in device
// memory that is part of the loaded library, so a call allocates nothing. It
// serves callers that must not allocate device memory while they run: an
// engine that sizes all of its device memory once at start-up (as VMLM sizes
// its pools at load) cannot have a library call cudaMalloc in its per-token
// loop, where the allocation could fail for lack of headroom and where
// cudaMalloc/cudaFree would also stall the loop by synchronising the device.
//
// Limits (the array is sized for decode): m <= 16 tokens, n <= 131072 output
// rows, k <= 16384. The array is kNaBytes (about 4.7 MB) and every GPU that
// loads the library holds it until the process exits.

namespace {

constexpr int kNaMaxM = 16;
constexpr int kNaMaxN = 131072;
constexpr int kNaMaxK = 16384;
constexpr int kNaMaxCtas = 160;  // grid cap; a B200 has 148 SMs
constexpr int kNaBn = 48;        // UMMA N for up to 16 tokens (3 planes x 16)
constexpr size_t kNaAlign(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }
constexpr size_t kNaErrOff = 0;                                        // int error word
constexpr size_t kNaCountersOff = 256;                                 // int32 per 128-row tile
constexpr size_t kNaMetaOff = kNaAlign(kNaCountersOff + 4 * (kNaMaxN / kTileRows));  // exps[16], flags[16]
constexpr size_t kNaSlotsOff = kNaAlign(kNaMetaOff + 2 * kNaMaxM * 4);
constexpr size_t kNaSlotsBytes = static_cast<size_t>(kNaMaxCtas) * kTileRows * kNaBn * 4;
constexpr size_t kNaPlanesOff = kNaAlign(kNaSlotsOff + kNaSlotsBytes);  // everything before starts at zero
constexpr size_t kNaPlanesBytes = static_cast<size_t>(3) * kNaMaxM * kNaMaxK;
constexpr size_t kNaBytes = kNaPlanesOff + kNaPlanesBytes;

}  // namespace

// The scratch itself. In host code this name is only a stand-in for the
// symbol: the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNaBytes];

namespace {

struct NaDevice {
  bool ready = false;
  unsigned char* base = nullptr;  // device address of g_noalloc_scratch on this device
  int sms = 0;
};
NaDevice g_na[64];

// One-time set-up per device, with that device current: resolve the array's
// device address, zero the part that must start at zero (error word,
// counters, split-tile slots; the kernels leave them zero after every call),
// and allow the GEMM kernel its shared memory. Allocates nothing.
int na_setup(int dev, NaDevice** out) {
  if (dev < 0 || dev >= 64) return fail(VMLM_ERR_ARG, "gemm_nt_int8_dev_noalloc: device %d out of range", dev);
  NaDevice& d = g_na[dev];
  if (!d.ready) {
    int major = 0, sms = 0;
    VMLM_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10) return fail(VMLM_ERR_NO_DEVICE, "device %d is not sm_100", dev);
    VMLM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    VMLM_TRY(load_encoder());
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(VMLM_ERR_CUDA, "gemm_nt_int8_dev_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    VMLM_CUDA(cudaMemset(ptr, 0, kNaPlanesOff));
    VMLM_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<TcMode::kQ8Swap>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kMaxSmem));
    d.base = static_cast<unsigned char*>(ptr);
    d.sms = sms < kNaMaxCtas ? sms : kNaMaxCtas;
    d.ready = true;
  }
  *out = &d;
  return VMLM_OK;
}

bool na_ready(int dev) { return dev >= 0 && dev < 64 && g_na[dev].ready; }

// The allocation-free calls record a kernel's bounded-wait timeout in the
// array's own error word. Read it after the whole device is idle (those calls
// may run on any stream); on an error, clear the word together with the
// split-tile counters and slots, which an aborted launch can leave non-zero
// and which every later call would otherwise sum into. Allocates nothing.
int na_take_error(int dev, int* code) {
  *code = 0;
  if (!na_ready(dev)) return VMLM_OK;
  NaDevice& d = g_na[dev];
  VMLM_CUDA(cudaDeviceSynchronize());
  int v = 0;
  VMLM_CUDA(cudaMemcpy(&v, d.base + kNaErrOff, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) {
    VMLM_CUDA(cudaMemset(d.base, 0, kNaPlanesOff));
    VMLM_CUDA(cudaDeviceSynchronize());
    *code = v;
  }
  return VMLM_OK;
}

}  // namespace

extern "C" int vmlm_gemm_nt_int8_dev_noalloc(const float* a, const int8_t* q, const float* scale, float* c,
                                             size_t m, size_t n, size_t k, void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  VMLM_TRY(check_dims(m, n, k));
  if (m == 0 || n == 0) return VMLM_OK;
  if (!c || !scale || (k > 0 && (!a || !q))) return fail(VMLM_ERR_ARG, "gemm_nt_int8_dev_noalloc: null pointer");
  if (m > static_cast<size_t>(kNaMaxM) || n > static_cast<size_t>(kNaMaxN) || k > static_cast<size_t>(kNaMaxK))
    return fail(VMLM_ERR_SHAPE,
                "gemm_nt_int8_dev_noalloc: m=%zu n=%zu k=%zu exceeds the fixed scratch limits m <= %d, n <= %d, "
                "k <= %d; use vmlm_gemm_nt_int8_dev",
                m, n, k, kNaMaxM, kNaMaxN, kNaMaxK);
  int dev = -1;
  VMLM_CUDA(cudaGetDevice(&dev));
  NaDevice* d = nullptr;
  VMLM_TRY(na_setup(dev, &d));
  cudaStream_t st = static_cast<cudaStream_t>(stream);  // NULL = the CUDA default stream
  const int M = static_cast<int>(m), N = static_cast<int>(n), K = static_cast<int>(k);
  const int kp = K > 0 ? static_cast<int>(cdiv(K, 16) * 16) : 16;
  int8_t* planes = reinterpret_cast<int8_t*>(d->base + kNaPlanesOff);
  int* exps = reinterpret_cast<int*>(d->base + kNaMetaOff);
  int* nonf = exps + kNaMaxM;
  VMLM_TRY(launch(q8_planes_kernel, dim3(M), dim3(kPrepThreads), 0, st, true, a, static_cast<long long>(K), M, K,
                  kp, planes, exps, nonf));
  const bool tc_ok = K > 0 && K % 16 == 0 && aligned16(q);
  if (!tc_ok) {
    const long long warps = static_cast<long long>(M) * N;
    return launch(q8_generic_kernel, dim3(static_cast<unsigned>(cdiv(warps * 32, 256))), dim3(256), 0, st, true, q,
                  scale, static_cast<const int8_t*>(planes), kp, static_cast<const int*>(exps),
                  static_cast<const int*>(nonf), a, static_cast<long long>(K), c, static_cast<long long>(N), M, N, K);
  }
  TcParams p = {};
  p.rows = N;
  p.cols = 3 * M;
  p.bn = kNaBn;
  p.kb_per_term = static_cast<int>(cdiv(K, 128));
  p.max_terms = 1;
  p.tiles_m = static_cast<int>(cdiv(N, kTileRows));
  p.tiles_n = 1;
  p.tm_fastest = 0;
  p.a_box_elems = 128;
  p.out = c;
  p.ldo = N;
  p.scale = scale;
  p.exps = exps;
  p.nonfinite = nonf;
  p.n_tokens = M;
  p.tok_per_tile = kNaBn / 3;
  p.n_out = N;
  p.x = a;
  p.ldx = K;
  p.w = q;
  p.k = K;
  p.slots = reinterpret_cast<uint32_t*>(d->base + kNaSlotsOff);
  p.counters = reinterpret_cast<int*>(d->base + kNaCountersOff);
  p.err = reinterpret_cast<int*>(d->base + kNaErrOff);
  int stages = 16;
  while (stages >= 2 && tc_smem_layout(stages, p.bn).total > static_cast<uint32_t>(kMaxSmem)) --stages;
  p.stages = stages;
  p.tmem_cols = pow2_at_least(2 * p.bn);
  const long long tiles = p.tiles_m;
  p.streamk = use_streamk(p, d->sms) ? 1 : 0;
  long long grid = p.streamk ? tiles * p.kb_per_term : tiles;
  if (grid > d->sms) grid = d->sms;
  CUtensorMap ma, mb;
  VMLM_TRY(make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, K, N, K, 128, kTileRows));
  VMLM_TRY(make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, planes, K, 3ull * M, kp, 128, p.bn));
  const TcSmem L = tc_smem_layout(stages, p.bn);
  return launch(tc_gemm_kernel<TcMode::kQ8Swap>, dim3(static_cast<unsigned>(grid)), dim3(kThreads), L.total, st, true,
                ma, mb, p);
}
