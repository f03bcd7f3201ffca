// decode_sk.cuh -- grouped Q8 decode with an equal share of weight bytes per
// CTA (stream-K over k-blocks), for batches of independent calls that have
// more 128-row tiles than the GPU has SMs.
//
// The one-CTA-per-tile grouped launch (q8_decode_kernel<DecGroup>) runs such a
// batch in two waves: a decoder layer's q/k/v/o/gate/up/down at m = 1 has 162
// tiles of K = 2304 and 18 of K = 5760 for 148 SMs, so 32 tiles and the long
// ones stream after the first wave has ended, from fewer SMs than HBM needs.
// Here the k-blocks of every tile, problem after problem and tile after tile,
// are cut into `grid` contiguous ranges of (almost) equal length, one per CTA,
// and every CTA streams its range without a second wave. A range covers the
// end of one tile, whole tiles and the start of another: up to kDecSkMaxSeg
// segments, each with its own TMEM accumulator, its own digit planes (made
// over the segment's K range, an exponent per token and segment) and its own
// epilogue.
//
//   warp 0      streams the range's W k-blocks (TMA, one tensor map per
//               problem) through a stage ring, segment after segment.
//   warps 2..9  make the digit planes of every segment (one register batch of
//               x chunks), or in planes mode load them from the planes
//               kernel's output (one exponent per token over the problem's
//               whole K), then run the segments' epilogues in order.
//   warp 1      owns TMEM; tcgen05.mma kind::i8 per k-block into the
//               segment's accumulator; a commit per segment.
//
// A segment that is a whole tile is written as a one-CTA tile of the grouped
// kernel writes it. A partial segment adds its f64 partials v_t * 2^-e into
// the tile's slot (atomicAdd at L2), then counts itself in the tile's counter
// (after a fence); the CTA whose count completes the tile reads the slot,
// rounds to f32, applies scale[n], stores C and clears slot and counter for
// the next call. No CTA waits for another. A token with NaN/Inf in a segment
// adds a NaN partial; the finishing CTA recomputes its outputs by sequential
// f32 dot products, as the other kernels do.
//
// Trace (vmlm_trace_enable): slots 0-7 as in the other kernels (start, planes
// ready, last W load issued, first stage consumed, last commit, first
// accumulator, epilogue done, TMEM released); slots 8-10 hold timestamps:
// first W load issued, plane warps past the wait for the previous kernel, and
// the CTA-wide set-up barrier passed.
//
// The partials of one output are integers times powers of two; their sum is
// exact in f64 (and so independent of the order of the atomic adds) while the
// segments' exponents of a token lie within 2^10 of each other, which holds
// for any activation row whose per-range maxima do. Every mbarrier wait is
// bounded.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "decode.cuh"
#include "ptx.cuh"

namespace vmlm {

constexpr int kDecSkMaxSeg = 4;

struct DecSkParams {
  int m;
  // 0: the kernel makes the digit planes. 1 (planes mode): the planes,
  // exponents and non-finite flags come from q8_planes_group_kernel (each
  // problem's map_p, exps, nonfinite: one exponent per token over the
  // problem's whole K), and each k-block's planes are loaded into the ring
  // stage of its W box
  int planes_mode;
  int rows_b;          // UMMA N: plane rows, 16 * ceil(3m / 16)
  int stages;          // W stage ring depth
  int kps;             // k-blocks per stage (1..3): a stage holds up to kps consecutive k-blocks of one segment;
                       // full ones arrive by one 3-D load (DecProblem::map3), shorter ones by 2-D loads
  int tmem_cols;       // kDecSkMaxSeg accumulators of rows_b columns, rounded up to a power of two
  int kbr_max;         // longest k-block range of one CTA
  int grid;            // CTAs; CTA b takes k-blocks [b * kb_total / grid, (b + 1) * kb_total / grid)
  long long kb_total;  // k-blocks of every tile of the batch
  double* slots;       // [tiles of the batch][m][128] f64 partial sums, zero between calls
  int* counters;       // [tiles of the batch] partial segments counted, zero between calls
  int* err;
  unsigned long long* trace;  // optional, kTraceSlots values per CTA
};

struct DecSkSmem {
  uint32_t stage, b_off, bar_off, meta_off, total;
};

__host__ __device__ inline DecSkSmem dec_sk_smem_layout(int stages, int rows_b, int kbr, int planes_mode,
                                                        int kps = 1) {
  DecSkSmem s;
  // a ring stage: kps W boxes, then in planes mode their k-blocks' planes;
  // the planes the kernel makes itself follow the ring
  s.stage = static_cast<uint32_t>(kps) *
            (kDecStageBytes + (planes_mode ? static_cast<uint32_t>(rows_b) * kBlockBytes : 0u));
  s.b_off = static_cast<uint32_t>(stages) * s.stage;  // the ring first, from offset 0
  s.bar_off = s.b_off + (planes_mode ? 0u : static_cast<uint32_t>(kbr) * rows_b * kBlockBytes);
  // full[stages], empty[stages], planes, tfull[kDecSkMaxSeg], done, drain; then the TMEM address and an abort word
  s.meta_off = s.bar_off + (2 * stages + 3 + kDecSkMaxSeg) * 8 + 16;
  // per segment and token: max |x| bits, non-finite flag, exponent; per segment: the finishing flag
  s.total = s.meta_off + (3 * kDecSkMaxSeg * kDecMaxTok + kDecSkMaxSeg) * 4 + 1024;
  return s;
}

// CTA whose k-block range holds global k-block x: the largest b with
// floor(b * total / grid) <= x.
__host__ __device__ inline int dec_sk_cta_of(long long x, long long total, int grid) {
  return static_cast<int>(((x + 1) * grid + total - 1) / total) - 1;
}

// The segments of CTA b's range: problem, tile of the problem, k-blocks
// [lo, hi) of the tile, first local k-block (j0 of unused entries is past
// every k-block). Returns false when the range needs more than kDecSkMaxSeg
// segments (the host plans only launches where no range does).
struct DecSkSegs {
  int n;
  int g[kDecSkMaxSeg], tile[kDecSkMaxSeg], lo[kDecSkMaxSeg], hi[kDecSkMaxSeg], j0[kDecSkMaxSeg];
};

template <class Prob>
__host__ __device__ inline bool dec_sk_segments(const Prob* prob, int count, long long total, int grid, int b,
                                                DecSkSegs& s) {
  const long long lo = static_cast<long long>(b) * total / grid;
  const long long hi = static_cast<long long>(b + 1) * total / grid;
  s.n = 0;
  long long x = lo;
  #pragma unroll
  for (int i = 0; i < kDecSkMaxSeg; ++i) {
    s.g[i] = 0;
    s.tile[i] = 0;
    s.lo[i] = 0;
    s.hi[i] = 0;
    s.j0[i] = 1 << 30;
    if (x < hi) {
      int g = 0;
      while (g + 1 < count && prob[g + 1].kbase <= x) ++g;
      const long long off = x - prob[g].kbase;
      const int t = static_cast<int>(off / prob[g].kb);
      const int kbi = static_cast<int>(off - static_cast<long long>(t) * prob[g].kb);
      const long long tile_end = prob[g].kbase + static_cast<long long>(t + 1) * prob[g].kb;
      const long long end = tile_end < hi ? tile_end : hi;
      s.g[i] = g;
      s.tile[i] = t;
      s.lo[i] = kbi;
      s.hi[i] = kbi + static_cast<int>(end - x);
      s.j0[i] = static_cast<int>(x - lo);
      s.n = i + 1;
      x = end;
    }
  }
  return x == hi;
}

// Device form of dec_sk_segments for a whole warp (every lane gets the same
// result). The problems' first k-blocks and k-block counts are kernel
// parameters: lane i reads problem i's (one load per lane, all in flight
// together) and a ballot finds the problem of a k-block, so no chain of
// dependent parameter loads delays the first TMA of the range.
__device__ __forceinline__ void dec_sk_segments_warp(const DecGroup& grp, long long total, int grid, int b,
                                                     DecSkSegs& s) {
  const int lane = threadIdx.x & 31;
  const int count = grp.count;
  const long long kbase = lane < count ? grp.prob[lane].kbase : (1ll << 62);
  const int kbl = lane < count ? grp.prob[lane].kb : 1;
  const long long lo = static_cast<long long>(b) * total / grid;
  const long long hi = static_cast<long long>(b + 1) * total / grid;
  s.n = 0;
  long long x = lo;
  #pragma unroll
  for (int i = 0; i < kDecSkMaxSeg; ++i) {
    s.g[i] = 0;
    s.tile[i] = 0;
    s.lo[i] = 0;
    s.hi[i] = 0;
    s.j0[i] = 1 << 30;
    if (x < hi) {  // warp-uniform
      const int g = __popc(__ballot_sync(0xffffffffu, kbase <= x)) - 1;
      const long long base = __shfl_sync(0xffffffffu, kbase, g);
      const int kb = __shfl_sync(0xffffffffu, kbl, g);
      const long long off = x - base;
      const int t = static_cast<int>(off / kb);
      const int kbi = static_cast<int>(off - static_cast<long long>(t) * kb);
      const long long tile_end = base + static_cast<long long>(t + 1) * kb;
      const long long end = tile_end < hi ? tile_end : hi;
      s.g[i] = g;
      s.tile[i] = t;
      s.lo[i] = kbi;
      s.hi[i] = kbi + static_cast<int>(end - x);
      s.j0[i] = static_cast<int>(x - lo);
      s.n = i + 1;
      x = end;
    }
  }
}

// Segment of local k-block j (segments are contiguous and in order).
__device__ __forceinline__ int dec_sk_seg_of(const DecSkSegs& s, int j) {
  int r = 0;
  #pragma unroll
  for (int i = 1; i < kDecSkMaxSeg; ++i) r += (j >= s.j0[i]) ? 1 : 0;
  return r;
}

template <class T>
__device__ __forceinline__ T dec_sk_pick(const T (&a)[kDecSkMaxSeg], int i) {
  T r = a[0];
  #pragma unroll
  for (int q = 1; q < kDecSkMaxSeg; ++q)
    if (i == q) r = a[q];
  return r;
}

// The x fields of a range's segments, read from the kernel parameters once.
struct DecSkX {
  const float* x[kDecSkMaxSeg];
  long long ldx[kDecSkMaxSeg];
  int k[kDecSkMaxSeg];
  int vec[kDecSkMaxSeg];
};

// x chunk qi of this CTA's range (float4 of token t at local chunk cc), zeros
// past the problem's K.
__device__ __forceinline__ float4 dec_sk_load(const DecSkSegs& sg, const DecSkX& sx, int qi, int qpt) {
  const int t = qi / qpt;
  const int cc = qi - t * qpt;
  const int j = cc >> 5;
  const int s = dec_sk_seg_of(sg, j);
  const int k = (dec_sk_pick(sg.lo, s) + j - dec_sk_pick(sg.j0, s)) * kBlockBytes + (cc & 31) * 4;
  if (k >= dec_sk_pick(sx.k, s)) return make_float4(0.f, 0.f, 0.f, 0.f);
  return dec_load4(dec_sk_pick(sx.x, s) + static_cast<long long>(t) * dec_sk_pick(sx.ldx, s) + k,
                   dec_sk_pick(sx.vec, s) != 0);
}

__global__ void __launch_bounds__(kDecThreads, 1)
    q8_decode_sk_kernel(const DecSkParams p, const __grid_constant__ DecGroup grp) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  const DecSkSmem L = dec_sk_smem_layout(p.stages, p.rows_b, p.kbr_max, p.planes_mode, p.kps);
  const uint32_t planes_slot0 = static_cast<uint32_t>(p.kps) * kDecStageBytes;  // a stage's planes, after its W
  const uint32_t planes_kb = static_cast<uint32_t>(p.rows_b) * kBlockBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty_bar = full_bar + p.stages;
  uint64_t* planes_bar = empty_bar + p.stages;
  uint64_t* tfull_bar = planes_bar + 1;  // [kDecSkMaxSeg]
  uint64_t* done_bar = tfull_bar + kDecSkMaxSeg;
  uint64_t* drain_bar = done_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_max = reinterpret_cast<int*>(smem + L.meta_off);  // [seg][kDecMaxTok]
  int* s_bad = s_max + kDecSkMaxSeg * kDecMaxTok;
  int* s_exp = s_bad + kDecSkMaxSeg * kDecMaxTok;
  volatile int* s_fin = s_exp + kDecSkMaxSeg * kDecMaxTok;  // [seg]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  DecSkSegs sg;
  dec_sk_segments_warp(grp, p.kb_total, p.grid, static_cast<int>(blockIdx.x), sg);
  const long long r_lo = static_cast<long long>(blockIdx.x) * p.kb_total / p.grid;
  const int nkb = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.kb_total / p.grid - r_lo);
  unsigned long long* trace = p.trace ? p.trace + static_cast<long long>(blockIdx.x) * kTraceSlots : nullptr;
  if (trace && threadIdx.x == 0) trace[0] = globaltimer();

  // x is on the critical path to the first MMA: the plane warps send their
  // loads first (after the previous kernel in the stream has finished).
  const int et = threadIdx.x - 64;  // plane/epilogue thread index, 0..255
  const int qpt = nkb * (kBlockBytes / 4);  // float4 chunks per token (a multiple of 32)
  const int nq = p.m * qpt;
  const int nsteps = (nq + kDecEpiThreads - 1) / kDecEpiThreads;  // <= kDecRegChunks (host rule)
  float4 keep[kDecRegChunks];
  if (warp >= 2) {
    DecSkX sx;
    #pragma unroll
    for (int i = 0; i < kDecSkMaxSeg; ++i) {
      const DecProblem& pr = grp.prob[sg.g[i]];
      sx.x[i] = pr.x;
      sx.ldx[i] = pr.ldx;
      sx.k[i] = pr.k;
      sx.vec[i] = pr.vec_x;
    }
    pdl_wait_prior();
    if (trace && et == 0) trace[9] = globaltimer();
    #pragma unroll
    for (int r = 0; r < (p.planes_mode ? 0 : kDecRegChunks); ++r) {
      const int qi = et + r * kDecEpiThreads;
      keep[r] = (r < nsteps && qi < nq) ? dec_sk_load(sg, sx, qi, qpt) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  // W producer state (thread 0). The first W loads are issued right after
  // the barriers are initialised, before the CTA-wide barrier below: the
  // weight stream does not wait for the other warps' set-up. Stage o
  // holds the k-blocks [j, j + n) of one segment (n <= kps): the range's
  // segments cut into runs of kps, the last run of each segment shorter.
  const uint64_t pol = policy_evict_first();
  int pstage = 0, pj = 0, nops = 0;
  uint32_t pphase = 0, issued_mask = 0, last_phase = 0;
  bool planes_ok = false;  // planes mode: the planes kernel has finished (loads may read its planes)
  // planes of stage `st` holding local k-blocks [j, j + n) of segment s
  auto issue_planes = [&](int st, int s, int j, int n) {
    const int kb = dec_sk_pick(sg.lo, s) + j - dec_sk_pick(sg.j0, s);
    for (int v = 0; v < n; ++v)
      tma_load_2d(smem + st * L.stage + planes_slot0 + v * planes_kb, &grp.prob[dec_sk_pick(sg.g, s)].map_p,
                  full_bar + st, (kb + v) * kBlockBytes, 0, policy_evict_last());
  };
  auto issue = [&]() {  // the stage that starts at local k-block pj
    const int s = dec_sk_seg_of(sg, pj);
    const int j1 = dec_sk_pick(sg.j0, s) + dec_sk_pick(sg.hi, s) - dec_sk_pick(sg.lo, s);
    const int n = min(p.kps, j1 - pj);
    const int kb = dec_sk_pick(sg.lo, s) + pj - dec_sk_pick(sg.j0, s);
    const DecProblem& pr = grp.prob[dec_sk_pick(sg.g, s)];
    const int row = dec_sk_pick(sg.tile, s) * kTileRows;
    mbar_arrive_expect_tx(full_bar + pstage, n * (kDecStageBytes + (p.planes_mode ? planes_kb : 0u)));
    uint8_t* st = smem + pstage * L.stage;
    if (n > 1 && n == p.kps) {
      tma_load_3d(st, &pr.map3, full_bar + pstage, row, kb, pol);
    } else {
      for (int v = 0; v < n; ++v)
        tma_load_2d(st + v * kDecStageBytes, &pr.map, full_bar + pstage, (kb + v) * kBlockBytes, row, pol);
    }
    if (p.planes_mode && planes_ok) issue_planes(pstage, s, pj, n);
    pj += n;
    ++nops;
    if (trace && issued_mask == 0) trace[8] = globaltimer();
    issued_mask |= 1u << pstage;
    last_phase = (last_phase & ~(1u << pstage)) | (pphase << pstage);
    if (++pstage == p.stages) {
      pstage = 0;
      pphase ^= 1;
    }
  };
  if (threadIdx.x == 0) {
    tma_prefetch_desc(p.kps > 1 ? &grp.prob[sg.g[0]].map3 : &grp.prob[sg.g[0]].map);
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full_bar + s, 1);
      mbar_init(empty_bar + s, 1);
    }
    mbar_init(planes_bar, 1);
    for (int s = 0; s < kDecSkMaxSeg; ++s) mbar_init(tfull_bar + s, 1);
    mbar_init(done_bar, kDecEpiWarps);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    // two stages go out before the CTA barrier, the rest of the first ring
    // right after it (all stages are free): a longer loop here holds up the
    // other warps' set-up and, at one token, the digit pass (C3 batch m = 1
    // 16.6 -> 16.3 µs per step)
    while (pj < nkb && nops < (p.stages < 2 ? p.stages : 2)) issue();
    pdl_launch_dependents();
  }
  if (threadIdx.x == 32) {
    // the segments' maps (a segment's last stage may take the 2-D map)
    #pragma unroll
    for (int s = 0; s < kDecSkMaxSeg; ++s)
      if (s < sg.n) {
        if (s > 0 || p.kps > 1) tma_prefetch_desc(&grp.prob[sg.g[s]].map);
        if (p.kps > 1 && s > 0) tma_prefetch_desc(&grp.prob[sg.g[s]].map3);
      }
  }
  if (threadIdx.x >= 64 && threadIdx.x < 64 + kDecSkMaxSeg * kDecMaxTok) {
    s_max[threadIdx.x - 64] = 0;
    s_bad[threadIdx.x - 64] = 0;
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (trace && threadIdx.x == 0) trace[10] = globaltimer();

  if (warp == 0) {
    // ------------------------------------------------------ W producer
    if (lane == 0) {
      if (p.planes_mode) {
        // the planes of the first ring, whose W boxes went out before the
        // wait for the planes kernel (same stages, same full barriers)
        pdl_wait_prior();
        planes_ok = true;
        for (int o = 0, j = 0; o < nops; ++o) {  // replay the first ring's stages
          const int s = dec_sk_seg_of(sg, j);
          const int j1 = dec_sk_pick(sg.j0, s) + dec_sk_pick(sg.hi, s) - dec_sk_pick(sg.lo, s);
          const int n = min(p.kps, j1 - j);
          issue_planes(o, s, j, n);
          j += n;
        }
      }
      while (pj < nkb) {
        if (!mbar_wait(empty_bar + pstage, pphase ^ 1, p.err, abort_flag, kDevTimeoutEmpty)) break;
        issue();
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
        #pragma unroll 1
        for (int s = 0; s < sg.n && ok; ++s) {
          const int j0 = dec_sk_pick(sg.j0, s);
          const int j1 = j0 + dec_sk_pick(sg.hi, s) - dec_sk_pick(sg.lo, s);
          const uint32_t acc = tmem_base + static_cast<uint32_t>(s * p.rows_b);
          #pragma unroll 1
          for (int j = j0; j < j1; j += p.kps) {
            if (!mbar_wait(full_bar + stage, phase, p.err, abort_flag, kDevTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (trace && !issued) trace[3] = globaltimer();
            const int n = min(p.kps, j1 - j);
            const uint32_t st = smem_u32(smem + stage * L.stage);
            for (int v = 0; v < n; ++v) {
              const uint32_t a_addr = st + v * kDecStageBytes;
              const uint32_t b_addr = p.planes_mode ? st + planes_slot0 + v * planes_kb
                                                    : smem_u32(smem + L.b_off + (j + v) * p.rows_b * kBlockBytes);
              #pragma unroll
              for (uint32_t u = 0; u < 4; ++u)
                umma_i8(acc, umma_desc_sw128(a_addr + 32 * u), umma_desc_sw128(b_addr + 32 * u), idesc,
                        (j + v > j0 || u > 0) ? 1u : 0u);
            }
            issued = true;
            umma_commit(empty_bar + stage);
            if (++stage == p.stages) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (ok) umma_commit(tfull_bar + s);
        }
      }
      if (trace) trace[4] = globaltimer();
      if (issued && *abort_flag) {
        // Let in-flight MMAs finish before TMEM is released.
        umma_commit(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, abort_flag, kDevTimeoutDrain, false);
      }
    }
  } else {
    // ----------------------------------- digit planes, then the epilogues
    if (p.planes_mode) {
      // the producer loads the planes with the W boxes; here the problems'
      // exponents and flags
      if (et == 0) mbar_arrive(planes_bar);
      if (et < kDecSkMaxSeg * kDecMaxTok) {
        const int s = et / kDecMaxTok, t = et - s * kDecMaxTok;
        if (s < sg.n && t < p.m) {
          const DecProblem& pr = grp.prob[dec_sk_pick(sg.g, s)];
          s_exp[et] = __ldg(pr.exps + t);
          s_bad[et] = __ldg(pr.nonfinite + t);
        }
      }
      named_bar_sync(1, kDecEpiThreads);
      if (trace && et == 0) trace[1] = globaltimer();
    } else {
      // pass 1: per segment and token, max |x| and the non-finite flag (32
      // consecutive chunks are one k-block of one token: one segment)
      #pragma unroll
      for (int r = 0; r < kDecRegChunks; ++r) {
        const int qi = et + r * kDecEpiThreads;
        if (r >= nsteps || qi - lane >= nq) break;  // warp-uniform
        const float4 v = keep[r];
        float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        int bad = !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
        mx = warp_max(mx);
        bad = warp_or(bad);
        if (lane == 0) {
          const int t = (qi - lane) / qpt;
          const int s = dec_sk_seg_of(sg, ((qi - lane) - t * qpt) >> 5);
          atomicMax(s_max + s * kDecMaxTok + t, __float_as_int(mx));
          if (bad) atomicOr(s_bad + s * kDecMaxTok + t, 1);
        }
      }
      named_bar_sync(1, kDecEpiThreads);
      if (et < kDecSkMaxSeg * kDecMaxTok) {
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
      // rows) of the chunk's local k-block
      uint8_t* planes = smem + L.b_off;
      #pragma unroll
      for (int r = 0; r < kDecRegChunks; ++r) {
        const int qi = et + r * kDecEpiThreads;
        if (r >= nsteps || qi >= nq) break;
        const int t = qi / qpt;
        const int cc = qi - t * qpt;
        const int j = cc >> 5;
        const int si = dec_sk_seg_of(sg, j) * kDecMaxTok + t;
        const float4 v = s_bad[si] ? make_float4(0.f, 0.f, 0.f, 0.f) : keep[r];
        const int e = s_exp[si];
        uint32_t w3[3];
        q8_digits4(v, e, w3[0], w3[1], w3[2]);
        const int b = (cc & 31) * 4;
        uint8_t* blk = planes + j * p.rows_b * kBlockBytes;
        #pragma unroll
        for (int pl = 0; pl < 3; ++pl) {
          const int row = 3 * t + pl;
          *reinterpret_cast<uint32_t*>(blk + row * kBlockBytes + ((((b >> 4) ^ (row & 7)) << 4) | (b & 15))) = w3[pl];
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, kDecEpiThreads);
      if (et == 0) {
        mbar_arrive(planes_bar);
        if (trace) trace[1] = globaltimer();
      }
    }

    // ------------------------------------------------------------ epilogues
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int t0 = half * 16;
    const int mt = p.m - t0 < 16 ? p.m - t0 : 16;  // tokens of this warp (may be <= 0)
    // scales are read while the MMAs run: this thread's row of a whole-tile
    // segment, and the row it finishes of a split tile (et mod 128 for every
    // token, as the finishing loop steps by 256)
    float sc_w[kDecSkMaxSeg], sc_f[kDecSkMaxSeg];
    #pragma unroll
    for (int i = 0; i < kDecSkMaxSeg; ++i) {
      const DecProblem& pr = grp.prob[sg.g[i]];
      const int nw = sg.tile[i] * kTileRows + row, nf = sg.tile[i] * kTileRows + (et & (kTileRows - 1));
      sc_w[i] = (i < sg.n && nw < pr.n) ? __ldg(pr.scale + nw) : 0.f;
      sc_f[i] = (i < sg.n && nf < pr.n) ? __ldg(pr.scale + nf) : 0.f;
    }
    bool all = true;
    #pragma unroll 1
    for (int s = 0; s < sg.n; ++s) {
      const DecProblem& pr = grp.prob[dec_sk_pick(sg.g, s)];
      const int tile = dec_sk_pick(sg.tile, s);
      const int n = tile * kTileRows + row;
      const bool whole = dec_sk_pick(sg.lo, s) == 0 && dec_sk_pick(sg.hi, s) == pr.kb;
      const float sc_row = dec_sk_pick(sc_w, s);
      const float sc_fin = dec_sk_pick(sc_f, s);
      uint32_t v[48];
      // Split tile: one thread reads (acquire) how many of the tile's other
      // parts are in its slot, before this segment's accumulator is ready.
      // When all are (usually this CTA's last segment, whose other parts sit
      // at the start of the next CTAs' ranges), their sum is final and each
      // thread loads its row's slot values while the MMAs finish.
      const long long gt = pr.tile0 + tile;
      double* slot = p.slots + gt * p.m * kTileRows;
      const long long kb_first = pr.kbase + static_cast<long long>(tile) * pr.kb;
      const int parts = dec_sk_cta_of(kb_first + pr.kb - 1, p.kb_total, p.grid) -
                        dec_sk_cta_of(kb_first, p.kb_total, p.grid) + 1;
      double pre[16];
      if (!whole) {
        if (et == 0) s_fin[s] = ld_acquire_gpu(p.counters + gt) == parts - 1 ? 2 : 0;
        named_bar_sync(1, kDecEpiThreads);
        #pragma unroll
        for (int jt = 0; jt < 16; ++jt)
          pre[jt] = (s_fin[s] == 2 && jt < mt && n < pr.n) ? __ldcg(slot + (t0 + jt) * kTileRows + row) : 0.0;
      }
      const bool have = all && mbar_wait(tfull_bar + s, 0, p.err, abort_flag, kDevTimeoutAccum, false);
      all = have;
      tc_fence_after();
      if (trace && et == 0 && s == 0) trace[5] = globaltimer();
      if (have && mt > 0) {
        const int nld = (3 * mt + 15) / 16;
        const uint32_t ta =
            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(s * p.rows_b + 3 * t0);
        tmem_ld16(ta, *reinterpret_cast<uint32_t(*)[16]>(v));
        if (nld > 1) tmem_ld16(ta + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
        if (nld > 2) tmem_ld16(ta + 32, *reinterpret_cast<uint32_t(*)[16]>(v + 32));
        tmem_ld_wait();
      }
      tc_fence_before();
      const int* sx = s_exp + s * kDecMaxTok;
      const int* sb = s_bad + s * kDecMaxTok;
      if (whole) {
        if (have && n < pr.n) {
          #pragma unroll
          for (int jt = 0; jt < 16; ++jt) {
            if (jt >= mt) break;
            const int t = t0 + jt;
            float r;
            if (sb[t]) {
              r = nonfinite_dot_q8(pr.x + static_cast<long long>(t) * pr.ldx, pr.w + static_cast<long long>(n) * pr.k,
                                   pr.k, sc_row);
            } else {
              const long long a = static_cast<long long>(static_cast<int>(v[3 * jt])) +
                                  256ll * static_cast<int>(v[3 * jt + 1]) + 65536ll * static_cast<int>(v[3 * jt + 2]);
              const int e = sx[t];
              if (e >= -70 && e <= 100)
                r = __fmul_rn(__fmul_rn(__ll2float_rn(a), __int_as_float((127 - e) << 23)), sc_row);
              else
                r = __fmul_rn(__double2float_rn(static_cast<double>(a) * pow2_f64(-e)), sc_row);
            }
            pr.out[static_cast<long long>(t) * pr.ldo + n] = r;
          }
        }
        continue;
      }
      // partial segment. When every other part was counted (s_fin 2), this
      // CTA finishes the tile from the slot values loaded above and its own
      // partials (in registers), without publishing them. Otherwise it adds
      // its f64 partials into the slot and counts them; the CTA whose count
      // completes the tile finishes it. f64 sums of the partials are exact,
      // so the order of the additions does not change the result. The
      // barriers run whatever the waits returned (after a failed wait the
      // results are invalid and the host clears slots and counters), so every
      // epilogue thread takes the same barriers.
      // this thread's partial of token t0 + jt (row `row`); NaN marks a recompute
      auto own = [&](int jt) -> double {
        const int t = t0 + jt;
        if (!have || sb[t]) return __longlong_as_double(0x7ff8000000000000ll);
        const long long a = static_cast<long long>(static_cast<int>(v[3 * jt])) +
                            256ll * static_cast<int>(v[3 * jt + 1]) + 65536ll * static_cast<int>(v[3 * jt + 2]);
        return static_cast<double>(a) * pow2_f64(-sx[t]);
      };
      if (s_fin[s] == 0) {
        if (have && n < pr.n) {
          #pragma unroll
          for (int jt = 0; jt < 16; ++jt) {
            if (jt >= mt) break;
            atomicAdd(slot + (t0 + jt) * kTileRows + row, own(jt));
          }
        }
        // the CTA barrier, then one acq_rel RMW by one thread: it releases the
        // whole CTA's adds (cumulative through the barrier) and, for the
        // finishing CTA, acquires the other CTAs' adds for the reads below
        named_bar_sync(1, kDecEpiThreads);
        if (et == 0) s_fin[s] = atom_add_acq_rel_gpu(p.counters + gt, 1) == parts - 1 ? 1 : 0;
        named_bar_sync(1, kDecEpiThreads);
      }
      if (s_fin[s] == 2) {
        // the last part: each thread finishes its own row's tokens
        if (n < pr.n) {
          #pragma unroll
          for (int jt = 0; jt < 16; ++jt) {
            if (jt >= mt) break;
            const int t = t0 + jt;
            const int idx = t * kTileRows + row;
            const double sum = pre[jt] + own(jt);
            float r;
            if (sum != sum)
              r = nonfinite_dot_q8(pr.x + static_cast<long long>(t) * pr.ldx, pr.w + static_cast<long long>(n) * pr.k,
                                   pr.k, sc_row);
            else
              r = __fmul_rn(__double2float_rn(sum), sc_row);
            pr.out[static_cast<long long>(t) * pr.ldo + n] = r;
            slot[idx] = 0.0;
          }
        }
        if (et == 0) p.counters[gt] = 0;
      } else if (s_fin[s] == 1) {
        for (int idx = et; idx < p.m * kTileRows; idx += kDecEpiThreads) {
          const int t = idx / kTileRows;
          const int nn = tile * kTileRows + (idx - t * kTileRows);
          if (nn < pr.n) {
            const double sum = __ldcg(slot + idx);
            float r;
            if (sum != sum)
              r = nonfinite_dot_q8(pr.x + static_cast<long long>(t) * pr.ldx, pr.w + static_cast<long long>(nn) * pr.k,
                                   pr.k, sc_fin);
            else
              r = __fmul_rn(__double2float_rn(sum), sc_fin);
            pr.out[static_cast<long long>(t) * pr.ldo + nn] = r;
            slot[idx] = 0.0;
          }
        }
        if (et == 0) p.counters[gt] = 0;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(done_bar);  // TMEM reads of this warp are complete
    if (trace && et == 0) trace[6] = globaltimer();
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
