// decode.cuh -- Q8 decode GEMM for few tokens (m <= 32) over few 128-row weight
// tiles: C[t][n] = f32(x[t,:] . f32(q[n,:])) * scale[n].
//
// One launch, no preparation kernel. A cluster of `c` CTAs owns one 128-row
// tile of W and splits its K range: CTA `rank` takes k-blocks [kb0, kb1).
//
//   warp 0      streams its W k-blocks (TMA, 128 x 128 bytes each) into a
//               stage ring; all of them are in flight before the kernel waits
//               for the previous kernel in the stream.
//   warps 2..9  read x[:, kb0*128 .. kb1*128) after that wait, pick a per-CTA
//               power-of-two exponent per token (e = 22 - E, max|x| = f*2^E
//               over this CTA's range), and write the three signed digit
//               planes of rint(x * 2^e) straight into shared memory in the
//               UMMA operand layout (K-major, 128-byte swizzle), row 3t+p.
//   warp 1      owns TMEM and issues tcgen05.mma kind::i8 (M = 128 W rows,
//               N = 16*ceil(3m/16) plane rows, s32 accumulators).
//   warps 2..9  then read the accumulator: v_t = a0 + 256 a1 + 65536 a2 is
//               exact in int64 and v_t * 2^-e exact in f64. With c == 1 the
//               CTA writes C directly. With c > 1 each CTA sends its f64
//               partials to the CTA that finishes those rows (rows are split
//               in c groups) through distributed shared memory; after one
//               cluster barrier every CTA sums its rows' partials in rank
//               order, rounds to f32 and applies scale[n].
//
// A token whose range holds NaN or Inf contributes a NaN partial; its outputs
// are recomputed by sequential f32 dot products (the same NaN/Inf outcome as
// any summation order). Every mbarrier wait is bounded.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "prep.cuh"
#include "ptx.cuh"
#include "tc_gemm.cuh"

namespace vmlm {

constexpr int kDecThreads = 320;
constexpr int kDecEpiWarps = 8;
constexpr int kDecEpiThreads = 32 * kDecEpiWarps;
constexpr int kDecMaxTok = 32;
constexpr int kDecMaxCluster = 8;
constexpr int kDecStageBytes = kTileRows * kBlockBytes;  // one 128 x 128 int8 W box
constexpr int kDecRegChunks = 8;                         // x float4 chunks per thread kept in registers
constexpr int kDecGroup = 4;                              // chunks per thread per rolled step of the digit pass

struct DecParams {
  int n, k, m;
  int kb;        // k-blocks of 128 bytes over K
  int cluster;   // CTAs that split one tile's K range
  int rows_b;    // UMMA N: plane rows, 16 * ceil(3m / 16)
  int kbr_max;   // largest k-block range of one CTA
  int stages;    // W stage ring depth
  int kps;       // k-blocks per W stage: 1 (2-D tensor maps) or 2..3 (3-D maps, one load per stage)
  int tmem_cols;
  int vec_x;     // x rows allow float4 loads
  // planes mode: the digit planes, exponents and non-finite flags come from
  // q8_planes_kernel (tmP maps its [3m][kp] planes) instead of being made here
  int planes_mode;
  const int* exps;
  const int* nonfinite;
  const float* x;
  long long ldx;
  const int8_t* w;
  const float* scale;
  float* out;
  long long ldo;
  int* err;
  unsigned long long* trace;  // optional, kTraceSlots values per CTA
};

// Grouped launches: independent Q8 calls with the same token count m run as one
// grid, a cluster of `cluster` CTAs per 128-row tile. Each problem carries its
// own weight tensor map, pointers and sizes; tile0 is its first tile (problems
// are listed by descending k, so the longest tiles start first).
struct DecProblem {
  CUtensorMap map;    // W [n][k] int8, box 128 x 128 (2-D), or 128 rows x kps k-blocks (3-D, kps > 1)
  CUtensorMap map_p;  // planes mode: the problem's planes [3m][kp], box 128 x rows_b
  CUtensorMap map3;   // q8_decode_sk_kernel with kps > 1: W as a 3-D map, box 128 rows x kps k-blocks
  const int* exps;
  const int* nonfinite;
  const float* x;
  const int8_t* w;
  const float* scale;
  float* out;
  long long ldx, ldo;
  long long kbase;  // equal-share launches (q8_decode_sk_kernel): first k-block of the problem over the batch
  int n, k, kb, tile0, vec_x;
};
constexpr int kDecMaxGroup = 16;
struct DecNoGroup {
  static constexpr int kMax = 0;
  int count;
};
struct DecGroup {
  static constexpr int kMax = kDecMaxGroup;
  DecProblem prob[kDecMaxGroup];
  int count;
};

// Rows of a tile finished by one CTA of the cluster.
__host__ __device__ inline int dec_rows_per_cta(int c) { return (kTileRows + c - 1) / c; }

struct DecSmem {
  uint32_t b_off, recv_off, bar_off, meta_off, total;
};

__host__ __device__ inline DecSmem dec_smem_layout(int stages, int rows_b, int kbr, int m, int c, int kps = 1) {
  DecSmem s;
  s.b_off = static_cast<uint32_t>(stages) * kps * kDecStageBytes;  // W stages first, from offset 0
  s.recv_off = s.b_off + static_cast<uint32_t>(kbr) * rows_b * kBlockBytes;
  const uint32_t recv = c > 1 ? static_cast<uint32_t>(c) * m * dec_rows_per_cta(c) * 8 : 0;
  s.bar_off = s.recv_off + ((recv + 15u) & ~15u);
  // full[stages], empty[stages], planes, tfull, done, drain, recv; then the TMEM address and an abort word
  s.meta_off = s.bar_off + (2 * stages + 5) * 8 + 16;
  // per token: max |x| bits, non-finite flag, exponent; then the scales of the rows this CTA finishes
  s.total = s.meta_off + 3 * kDecMaxTok * 4 + kTileRows * 4 + 1024;
  return s;
}

// 2^e as a double for |e| <= 1022 (the exponents here stay within [-170, 106]).
__device__ __forceinline__ double pow2_f64(int e) {
  return __longlong_as_double(static_cast<long long>(1023 + e) << 52);
}

__device__ __forceinline__ float4 dec_load4(const float* p, bool vec) {
  if (vec) return *reinterpret_cast<const float4*>(p);
  return make_float4(p[0], p[1], p[2], p[3]);
}

// One batch of x chunks for the digit planes: chunk (s0 + r) * 256 + et of this
// CTA's range, r < kDecRegChunks (zeros past the range or past K).
__device__ __forceinline__ void dec_load_batch(const DecParams& p, float4 (&keep)[kDecRegChunks], int s0, int et,
                                               int k_lo, int qpt, int nq, int nsteps, bool vec) {
  #pragma unroll
  for (int r = 0; r < kDecRegChunks; ++r) {
    const int qi = et + (s0 + r) * kDecEpiThreads;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s0 + r < nsteps && qi < nq) {
      const int t = qi / qpt;
      const int k = k_lo + (qi - t * qpt) * 4;
      if (k < p.k) v = dec_load4(p.x + static_cast<long long>(t) * p.ldx + k, vec);
    }
    keep[r] = v;
  }
}

// Exact f32 recompute of one output of a token that holds NaN or Inf (out of
// line: see nonfinite_dot_q8).
__device__ __forceinline__ float dec_nonfinite_dot(const DecParams& p, int t, int n) {
  return nonfinite_dot_q8(p.x + static_cast<long long>(t) * p.ldx, p.w + static_cast<long long>(n) * p.k, p.k,
                          __ldg(p.scale + n));
}

// Issue W stage `stage`: the ops index o covers k-blocks [kb0 + o * kps, +kps)
// of the tile's 128 rows; the copy completes on the stage's full barrier.
__device__ __forceinline__ void dec_issue_w(const DecParams& p, const CUtensorMap* map_w, uint8_t* smem,
                                            uint64_t* full_bar, int stage, int o, uint32_t stage_bytes, int kb0,
                                            int tile, uint64_t pol) {
  mbar_arrive_expect_tx(full_bar + stage, stage_bytes);
  if (p.kps == 1)
    tma_load_2d(smem + stage * stage_bytes, map_w, full_bar + stage, (kb0 + o) * kBlockBytes, tile * kTileRows, pol);
  else  // k-blocks past this CTA's range are loaded (zeros past K) but not multiplied
    tma_load_3d(smem + stage * stage_bytes, map_w, full_bar + stage, tile * kTileRows, kb0 + o * p.kps, pol);
}

template <class G>
__global__ void __launch_bounds__(kDecThreads, 1)
    q8_decode_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmP,
                     const DecParams p_in, const __grid_constant__ G grp) {
  DecParams p = p_in;  // a grouped launch replaces the per-problem fields below
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  const DecSmem L = dec_smem_layout(p.stages, p.rows_b, p.kbr_max, p.m, p.cluster, p.kps);
  const uint32_t stage_bytes = static_cast<uint32_t>(p.kps) * kDecStageBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty_bar = full_bar + p.stages;
  uint64_t* planes_bar = empty_bar + p.stages;
  uint64_t* tfull_bar = planes_bar + 1;
  uint64_t* done_bar = tfull_bar + 1;
  uint64_t* drain_bar = done_bar + 1;
  uint64_t* recv_bar = drain_bar + 1;  // clusters: the partials of the rows this CTA finishes have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_max = reinterpret_cast<int*>(smem + L.meta_off);
  int* s_bad = s_max + kDecMaxTok;
  int* s_exp = s_bad + kDecMaxTok;
  float* s_scale = reinterpret_cast<float*>(s_exp + kDecMaxTok);
  double* recv = reinterpret_cast<double*>(smem + L.recv_off);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const CUtensorMap* map_w = &tmW;
  const CUtensorMap* map_p = &tmP;
  const int c = p.cluster;
  const int rank = c > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  int tile = blockIdx.x / c;
  if constexpr (G::kMax > 0) {
    // this cluster's problem: the last one whose first tile is at or before it
    int g = 0;
    while (g + 1 < grp.count && grp.prob[g + 1].tile0 <= tile) ++g;
    const DecProblem& pr = grp.prob[g];
    p.x = pr.x;
    p.ldx = pr.ldx;
    p.w = pr.w;
    p.scale = pr.scale;
    p.out = pr.out;
    p.ldo = pr.ldo;
    p.n = pr.n;
    p.k = pr.k;
    p.kb = pr.kb;
    p.vec_x = pr.vec_x;
    p.exps = pr.exps;
    p.nonfinite = pr.nonfinite;
    map_w = &pr.map;
    map_p = &pr.map_p;
    tile -= pr.tile0;
  }
  const int kb0 = static_cast<int>(static_cast<long long>(rank) * p.kb / c);
  const int kb1 = static_cast<int>(static_cast<long long>(rank + 1) * p.kb / c);
  const int nkb = kb1 - kb0;
  const int nops = (nkb + p.kps - 1) / p.kps;  // W stages of this CTA's range
  unsigned long long* trace = p.trace ? p.trace + static_cast<long long>(blockIdx.x) * kTraceSlots : nullptr;
  if (trace && threadIdx.x == 0) trace[0] = globaltimer();

  // x is on the critical path to the first MMA: the plane warps send their
  // first batch of x loads before anything else (after the previous kernel in
  // the stream, which may produce x, has finished).
  const int et = threadIdx.x - 64;  // plane/epilogue thread index, 0..255
  const int k_lo = kb0 * kBlockBytes;
  const int qpt = nkb * (kBlockBytes / 4);  // float4 chunks per token (a multiple of 32)
  const int nq = p.m * qpt;
  const int nsteps = (nq + kDecEpiThreads - 1) / kDecEpiThreads;
  const bool vec = p.vec_x != 0;
  float4 keep[kDecRegChunks];
  if (warp >= 2) {
    pdl_wait_prior();
    if (!p.planes_mode) dec_load_batch(p, keep, 0, et, k_lo, qpt, nq, nsteps, vec);
  }

  if (threadIdx.x == 0) {
    pdl_launch_dependents();
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full_bar + s, 1);
      mbar_init(empty_bar + s, 1);
    }
    mbar_init(planes_bar, 1);
    mbar_init(tfull_bar, 1);
    mbar_init(done_bar, kDecEpiWarps);
    mbar_init(drain_bar, 1);
    mbar_init(recv_bar, 1);
    if (c > 1) {
      // every CTA of the cluster sends one f64 partial per token for each row this CTA finishes
      const int rpc = dec_rows_per_cta(c);
      const int r_cnt = kTileRows - rank * rpc < rpc ? kTileRows - rank * rpc : rpc;
      mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>(c * p.m * (r_cnt > 0 ? r_cnt : 0) * 8));
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // The first W stages go out from this thread (the producer) right after it
  // has initialised their barriers, ahead of the CTA barrier below: the
  // weights are the bytes the call waits for, and their first stage no longer
  // waits for the TMEM allocation and the other warps' set-up.
  const int pre = nops < p.stages ? nops : p.stages;
  if (threadIdx.x == 0) {
    const uint64_t pol = policy_evict_first();
    for (int o = 0; o < pre; ++o) dec_issue_w(p, map_w, smem, full_bar, o, o, stage_bytes, kb0, tile, pol);
  }
  if (threadIdx.x >= 64 && threadIdx.x < 64 + kDecMaxTok) {
    s_max[threadIdx.x - 64] = 0;
    s_bad[threadIdx.x - 64] = 0;
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Cluster phase 1 (arrive now, wait before the first remote store): every
  // CTA of the cluster is running before any writes into another's memory.
  if (c > 1) cluster_arrive_relaxed();

  if (warp == 0) {
    // ------------------------------------------------------ W producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, last_phase = 0;
      for (int o = 0; o < nops; ++o) {
        if (o >= pre) {  // the first `pre` stages went out before the CTA barrier
          if (!mbar_wait(empty_bar + stage, phase ^ 1, p.err, abort_flag, kDevTimeoutEmpty)) break;
          dec_issue_w(p, map_w, smem, full_bar, stage, o, stage_bytes, kb0, tile, pol);
        }
        issued_mask |= 1u << stage;
        last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (trace) trace[2] = globaltimer();
      if (*abort_flag) {
        for (int s = 0; s < p.stages; ++s)
          if (issued_mask & (1u << s))
            mbar_wait(full_bar + s, (last_phase >> s) & 1u, nullptr, abort_flag, kDevTimeoutDrain, false);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(2, 1, kTileRows, p.rows_b);
      bool issued = false;
      if (mbar_wait(planes_bar, 0, p.err, abort_flag, kDevTimeoutFull)) {
        tc_fence_after();
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int o = 0; o < nops; ++o) {
          if (!mbar_wait(full_bar + stage, phase, p.err, abort_flag, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (trace && !issued) trace[3] = globaltimer();
          const int nv = min(p.kps, nkb - o * p.kps);
          for (int v = 0; v < nv; ++v) {
            const int j = o * p.kps + v;
            const uint32_t a_addr = smem_u32(smem + stage * stage_bytes + v * kDecStageBytes);
            const uint32_t b_addr = smem_u32(smem + L.b_off + j * p.rows_b * kBlockBytes);
            #pragma unroll
            for (uint32_t u = 0; u < 4; ++u)
              umma_i8(tmem_base, umma_desc_sw128(a_addr + 32 * u), umma_desc_sw128(b_addr + 32 * u), idesc,
                      (j > 0 || u > 0) ? 1u : 0u);
          }
          issued = true;
          umma_commit(empty_bar + stage);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(tfull_bar);
      }
      if (trace) trace[4] = globaltimer();
      if (issued && *abort_flag) {
        // Let in-flight MMAs finish before TMEM is released.
        umma_commit(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, abort_flag, kDevTimeoutDrain, false);
      }
    }
  } else {
    // ----------------------------------- digit planes, then the epilogue
    if (p.planes_mode) {
      // The planes come from q8_planes_kernel, the previous kernel in the
      // stream (waited for above): one TMA load per k-block of this CTA's
      // range, in the layout pass 2 below writes (128-byte swizzle, rows
      // past 3m read as zero), and the per-token exponents and flags.
      if (et == 0) {
        mbar_arrive_expect_tx(planes_bar, static_cast<uint32_t>(nkb * p.rows_b * kBlockBytes));
        for (int j = 0; j < nkb; ++j)
          tma_load_2d(smem + L.b_off + j * p.rows_b * kBlockBytes, map_p, planes_bar, (kb0 + j) * kBlockBytes, 0,
                      policy_evict_last());
        if (trace) trace[1] = globaltimer();
      }
      if (et < p.m) {
        s_exp[et] = __ldg(p.exps + et);
        s_bad[et] = __ldg(p.nonfinite + et);
      }
      named_bar_sync(1, kDecEpiThreads);
    } else {
      // pass 1: per-token max |x| and non-finite flag over this CTA's range, in
      // batches of kDecRegChunks chunks per thread whose loads are all in flight
      // before any is reduced; the first batch stays in registers for pass 2.
      // 32 consecutive chunks never straddle a token (qpt % 32 == 0).
      for (int s0 = 0; s0 < nsteps; s0 += kDecRegChunks) {
        if (s0 > 0) dec_load_batch(p, keep, s0, et, k_lo, qpt, nq, nsteps, vec);  // batch 0 is in flight
        #pragma unroll
        for (int r = 0; r < kDecRegChunks; ++r) {
          const int qi = et + (s0 + r) * kDecEpiThreads;
          if (s0 + r >= nsteps || qi - lane >= nq) break;  // warp-uniform
          const float4 v = keep[r];
          float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
          int bad = !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
          mx = warp_max(mx);
          bad = warp_or(bad);
          if (lane == 0) {
            const int t = (qi - lane) / qpt;
            atomicMax(s_max + t, __float_as_int(mx));
            if (bad) atomicOr(s_bad + t, 1);
          }
        }
      }
      const bool kept = nsteps <= kDecRegChunks;  // else pass 2 reloads (L2 hits)
      named_bar_sync(1, kDecEpiThreads);
      if (et < p.m) {
        int e = 0;
        const float amax = __int_as_float(s_max[et]);
        if (!s_bad[et] && amax > 0.f) {
          int E;
          frexpf(amax, &E);
          e = 22 - E;
        }
        s_exp[et] = e;
      }
      named_bar_sync(1, kDecEpiThreads);
      // pass 2: digits into the swizzled B tiles (row 3t+p, K-major, 128-byte
      // rows), in groups of kDecGroup chunks per thread: taken from the kept
      // batch when the range fits it, else loaded again (L2 hits) with the
      // group's loads in flight together. The loop stays rolled: its body is
      // the hot code of this phase and must stay small in the instruction cache.
      uint8_t* planes = smem + L.b_off;
      #pragma unroll 1
      for (int s0 = 0; s0 < nsteps; s0 += kDecGroup) {
        float4 g[kDecGroup];
        #pragma unroll
        for (int i = 0; i < kDecGroup; ++i) {
          const int s = s0 + i;
          const int qi = et + s * kDecEpiThreads;
          g[i] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (kept) {
            #pragma unroll
            for (int r = 0; r < kDecRegChunks; ++r)
              if (r == s) g[i] = keep[r];
          } else if (s < nsteps && qi < nq) {
            const int t = qi / qpt;
            const int k = k_lo + (qi - t * qpt) * 4;
            if (k < p.k) g[i] = dec_load4(p.x + static_cast<long long>(t) * p.ldx + k, vec);
          }
        }
        #pragma unroll
        for (int i = 0; i < kDecGroup; ++i) {
          const int qi = et + (s0 + i) * kDecEpiThreads;
          if (s0 + i >= nsteps || qi >= nq) break;
          const int t = qi / qpt;
          const int kk = (qi - t * qpt) * 4;  // offset in this CTA's range
          const float4 v = s_bad[t] ? make_float4(0.f, 0.f, 0.f, 0.f) : g[i];
          const int e = s_exp[t];
          uint32_t w3[3];
          q8_digits4(v, e, w3[0], w3[1], w3[2]);
          const int j = kk >> 7, b = kk & 127;
          uint8_t* blk = planes + j * p.rows_b * kBlockBytes;
          #pragma unroll
          for (int pl = 0; pl < 3; ++pl) {
            const int row = 3 * t + pl;
            *reinterpret_cast<uint32_t*>(blk + row * kBlockBytes + ((((b >> 4) ^ (row & 7)) << 4) | (b & 15))) =
                w3[pl];
          }
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, kDecEpiThreads);
      if (et == 0) {
        mbar_arrive(planes_bar);
        if (trace) trace[1] = globaltimer();
      }
    }

    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int n = tile * kTileRows + row;
    const int t0 = half * 16;
    const int mt = p.m - t0 < 16 ? p.m - t0 : 16;  // tokens of this warp (may be <= 0)
    const int rpc = dec_rows_per_cta(c);
    const int r_lo = rank * rpc;
    const int r_cnt = kTileRows - r_lo < rpc ? kTileRows - r_lo : rpc;
    // scales are read while the MMAs run
    const float sc_row = (c == 1 && n < p.n) ? __ldg(p.scale + n) : 0.f;
    if (c > 1 && et < r_cnt && tile * kTileRows + r_lo + et < p.n) s_scale[et] = __ldg(p.scale + tile * kTileRows + r_lo + et);
    uint32_t v[48];
    const bool have = mbar_wait(tfull_bar, 0, p.err, abort_flag, kDevTimeoutAccum, false);
    tc_fence_after();
    const unsigned long long t_acc = trace ? globaltimer() : 0;
    if (trace && et == 0) trace[5] = t_acc;
    if (have && mt > 0) {
      const int nld = (3 * mt + 15) / 16;
      const uint32_t ta = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + 3 * t0;
      tmem_ld16(ta, *reinterpret_cast<uint32_t(*)[16]>(v));
      if (nld > 1) tmem_ld16(ta + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
      if (nld > 2) tmem_ld16(ta + 32, *reinterpret_cast<uint32_t(*)[16]>(v + 32));
      tmem_ld_wait();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(done_bar);  // TMEM reads of this warp are complete
    if (trace && et == 0) trace[8] = globaltimer() - t_acc;

    if (c == 1) {
      if (have && n < p.n) {
        const float sc = sc_row;
        #pragma unroll
        for (int jt = 0; jt < 16; ++jt) {
          if (jt >= mt) break;
          const int t = t0 + jt;
          float r;
          if (s_bad[t]) {
            r = dec_nonfinite_dot(p, t, n);
          } else {
            const long long a = static_cast<long long>(static_cast<int>(v[3 * jt])) +
                                256ll * static_cast<int>(v[3 * jt + 1]) +
                                65536ll * static_cast<int>(v[3 * jt + 2]);
            const int e = s_exp[t];
            if (e >= -70 && e <= 100)
              r = __fmul_rn(__fmul_rn(__ll2float_rn(a), __int_as_float((127 - e) << 23)), sc);
            else
              r = __fmul_rn(__double2float_rn(static_cast<double>(a) * pow2_f64(-e)), sc);
          }
          p.out[static_cast<long long>(t) * p.ldo + n] = r;
        }
      }
    } else {
      const int owner = row / rpc;
      const int rl = row - owner * rpc;
      const uint32_t dst = mapa_shared(smem_u32(recv), static_cast<uint32_t>(owner));
      const uint32_t dst_bar = mapa_shared(smem_u32(recv_bar), static_cast<uint32_t>(owner));
      cluster_wait_acquire();  // phase 1: the owner CTA is running and its barriers are initialised
      if (trace && et == 0) trace[9] = globaltimer() - t_acc;
      #pragma unroll
      for (int jt = 0; jt < 16; ++jt) {
        if (jt >= mt) break;
        const int t = t0 + jt;
        double part;
        if (!have || s_bad[t]) {
          part = __longlong_as_double(0x7ff8000000000000ll);  // NaN marks a recompute
        } else {
          const long long a = static_cast<long long>(static_cast<int>(v[3 * jt])) +
                              256ll * static_cast<int>(v[3 * jt + 1]) + 65536ll * static_cast<int>(v[3 * jt + 2]);
          part = static_cast<double>(a) * pow2_f64(-s_exp[t]);
        }
        st_async_cluster_f64(dst + static_cast<uint32_t>(((rank * p.m + t) * rpc + rl) * 8), part, dst_bar);
      }
      if (trace && et == 0) trace[10] = globaltimer() - t_acc;
      // the partials of this CTA's rows from every CTA of the cluster (its own
      // included) have landed: no CTA writes into this one after this point
      const bool got = mbar_wait(recv_bar, 0, p.err, abort_flag, kDevTimeoutAccum, false);
      if (trace && et == 0) trace[11] = globaltimer() - t_acc;
      const int total = r_cnt > 0 ? p.m * r_cnt : 0;
      for (int idx = et; idx < total; idx += kDecEpiThreads) {
        const int t = idx / r_cnt;
        const int rr = idx - t * r_cnt;
        const int nn = tile * kTileRows + r_lo + rr;
        if (nn >= p.n) continue;
        double sum = 0.0;
        for (int q = 0; q < c; ++q) sum += recv[(q * p.m + t) * rpc + rr];
        if (!got) sum = __longlong_as_double(0x7ff8000000000000ll);
        float r;
        if (sum != sum)
          r = dec_nonfinite_dot(p, t, nn);
        else
          r = __fmul_rn(__double2float_rn(sum), s_scale[rr]);
        p.out[static_cast<long long>(t) * p.ldo + nn] = r;
      }
    }
    // planes mode after an abort: the planes copy must land before this
    // CTA's shared memory is released
    if (p.planes_mode && et == 0 && *abort_flag) mbar_wait(planes_bar, 0, nullptr, abort_flag, kDevTimeoutDrain, false);
    if (trace && et == 0) trace[6] = globaltimer();
  }

  // Warps 0 and 1 take the cluster step the epilogue warps took.
  if (warp < 2) {
    __syncwarp();
    if (c > 1) cluster_wait_acquire();
  }
  if (warp == 1) {
    mbar_wait(done_bar, 0, p.err, abort_flag, kDevTimeoutDrain, false);
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem_base, p.tmem_cols);
    if (trace && lane == 0) trace[7] = globaltimer();
  }
}

}  // namespace vmlm
