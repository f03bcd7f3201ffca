// tc2_gemm.cuh -- the prefill GEMM on CTA pairs (tcgen05 cta_group::2).
//
// For large normal-mode GEMMs (kI8Norm, kBf16Norm: A the activations, B the
// weight rows) and for Q8 calls with many weight tiles (kQ8Swap: A the weight
// rows, B the activation digit planes): C = A . B^T. A cluster of two CTAs
// owns a 256 x bn tile: CTA r holds A rows [256*tm + 128*r, +128) and B rows
// [bn*tn + (bn/2)*r, +bn/2) in its own shared memory (same offsets in both),
// and its 128 accumulator rows x bn columns in its own TMEM (same address).
// The even CTA issues tcgen05.mma.cta_group::2 with M = 256, N = bn. Per MAC
// each SM loads fewer operand bytes than a 128 x bn tile on one SM (B is
// split between the two), which is what bounds these GEMMs (per-SM L2 -> SM
// bandwidth; in swap mode the planes are re-read for every weight tile).
// kBf16Norm calls with few tiles split K in two (p.ksplit = 2): twice the
// pairs, half the operand bytes each, and each pair adds its partial into C
// (zeroed by the prep kernel) with red.global.add. f32 addition commutes, so
// the two partials give the same bits in either order.
//
// Warp roles as in tc_gemm_kernel (320 threads). Barriers:
//   full[s]   even CTA only: its producer expects both CTAs' bytes; both CTAs'
//             TMA loads complete on it (.cta_group::2 loads name it)
//   empty[s]  both CTAs: the even CTA's MMA commit arrives on both
//   tfull[b]  both CTAs: same
//   tempty[b] even CTA only: 8 local + 8 remote epilogue-warp arrivals
// Tiles are taken round-robin by pairs (persistent). Every wait is bounded;
// a final cluster barrier keeps both CTAs (and their shared memory and TMEM)
// alive until neither has work or remote arrivals left.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"
#include "tc_gemm.cuh"

namespace vmlm {

constexpr int kPairRows = 2 * kTileRows;

struct Tc2Smem {
  uint32_t a_off, b_off, bar_off, meta_off, stg_off;
  uint32_t a_bytes, b_bytes, total;
};

// a_bytes / b_bytes: one stage of each operand (kps k-blocks of 128 bytes per row)
__host__ __device__ inline Tc2Smem tc2_smem_layout(int stages, int bn, int kps = 1) {
  Tc2Smem s;
  s.a_bytes = static_cast<uint32_t>(kps) * kTileRows * kBlockBytes;
  s.b_bytes = static_cast<uint32_t>(kps) * static_cast<uint32_t>(bn / 2) * kBlockBytes;
  s.a_off = 0;
  s.b_off = s.a_off + stages * s.a_bytes;
  s.bar_off = s.b_off + stages * s.b_bytes;
  // full[stages], empty[stages], tfull[2], tempty[2], drain, done, then 64 bytes of words
  s.meta_off = s.bar_off + (2 * stages + 6) * 8 + 64;
  // column scales of a tile (bn <= 256 floats), or in swap mode the tile's
  // token exponents and flags (2 x 128 words)
  s.stg_off = s.meta_off + 256 * 4;
  s.total = s.stg_off + kEpiWarps * 32 * 17 * 4 + 1024;
  return s;
}

template <TcMode MODE>
__global__ void __launch_bounds__(kThreads, 1)
    tc2_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const TcParams p) {
  static_assert(MODE == TcMode::kI8Norm || MODE == TcMode::kBf16Norm || MODE == TcMode::kQ8Swap,
                "kI8Norm, kBf16Norm, kQ8Swap");
  constexpr bool kInt = (MODE == TcMode::kI8Norm || MODE == TcMode::kQ8Swap);
  constexpr bool kSwap = (MODE == TcMode::kQ8Swap);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  const Tc2Smem L = tc2_smem_layout(p.stages, p.bn, p.kps);
  const uint32_t a_kb_bytes = kTileRows * kBlockBytes;                         // one k-block of A
  const uint32_t b_kb_bytes = static_cast<uint32_t>(p.bn / 2) * kBlockBytes;  // one k-block of B
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty_bar = full_bar + p.stages;
  uint64_t* tfull_bar = empty_bar + p.stages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* done_bar = drain_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_scale = reinterpret_cast<float*>(smem + L.meta_off);
  int* s_exp = reinterpret_cast<int*>(s_scale);  // swap mode: tokens of a tile (<= 80)
  int* s_bad = s_exp + 128;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int tiles = p.tiles_m * p.tiles_n;
  uint32_t* s_stage = reinterpret_cast<uint32_t*>(smem + L.stg_off) + (warp >= 2 ? warp - 2 : 0) * 32 * 17;
  unsigned long long* trace = p.trace ? p.trace + static_cast<long long>(blockIdx.x) * kTraceSlots : nullptr;
  if (trace && threadIdx.x == 0) trace[0] = globaltimer();

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full_bar + s, 1);
      mbar_init(empty_bar + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar + b, 1);
      mbar_init(tempty_bar + b, 2 * kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    mbar_init(done_bar, kEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Both CTAs' barriers are initialised before any remote arrival or copy.
  cluster_arrive_release();
  cluster_wait_acquire();
  // The next kernel in the stream may be scheduled now: kernels this library
  // launches as programmatic dependents wait for this one to complete before
  // they touch memory it reads or writes (they only prefetch weights first).
  pdl_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_even = mapa_shared(smem_u32(full_bar), 0);
  const uint32_t tempty_even = mapa_shared(smem_u32(tempty_bar), 0);
  const int kbt = p.kb_per_term;

  // Work item i of this pair (round-robin over pairs): this CTA's 128 rows of
  // A start at a_row; tn is the column tile; k-blocks [kb0, kb1) of each term
  // (the whole K, or one of p.ksplit ranges: items [r*tiles, (r+1)*tiles) take
  // range r). Both CTAs see the same sequence.
  const int ks = p.ksplit > 1 ? p.ksplit : 1;
  auto tile_of = [&](int i, int& a_row, int& tn, int& kb0, int& kb1) -> bool {
    const int item = pair + i * npairs;
    if (item >= tiles * ks) return false;
    const int tile = item % tiles;
    const int r = item / tiles;
    tn = tile / p.tiles_m;
    a_row = (tile % p.tiles_m) * kPairRows + static_cast<int>(crank) * kTileRows;
    kb0 = r * kbt / ks;
    kb1 = (r + 1) * kbt / ks;
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      // Swap mode: the weights (A) stream once (evict first), the digit planes
      // (B) are re-read by every tile. Normal modes: both operands are re-read,
      // the activations by every column tile and a weight tile by every row
      // tile (C5: 16), so both are kept (evict last; C5 617-628 -> 603 us
      // against weights marked evict-first).
      const uint64_t pol_a = kSwap ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = policy_evict_last();
      uint32_t issued_mask = 0, last_phase = 0;
      unsigned long long wait_empty = 0;  // trace: time waiting for free stages
      // (issuing the weight half of the first stages before this wait, as the
      // one-CTA kernel does, delays the previous kernel in the stream here)
      pdl_wait_prior();
      const int T = (MODE == TcMode::kBf16Norm) ? active_terms(p) : 1;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int a_row, tn, kb0, kb1;
      for (int i = 0; ok && tile_of(i, a_row, tn, kb0, kb1); ++i) {
        const int b_row = tn * p.bn + static_cast<int>(crank) * (p.bn / 2);
        const int nops = (kb1 - kb0 + p.kps - 1) / p.kps;  // stages per term
        for (int j = 0; j < T * nops; ++j) {
          const int term = j / nops;
          const int kin = kb0 + (j - term * nops) * p.kps;
          const unsigned long long tw = trace ? globaltimer() : 0;
          if (!mbar_wait(empty_bar + stage, phase ^ 1, p.err, abort_flag, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (trace) wait_empty += globaltimer() - tw;
          if (crank == 0) mbar_arrive_expect_tx(full_bar + stage, 2 * (L.a_bytes + L.b_bytes));
          const uint32_t fb = full_even + stage * 8;
          if (p.kps == 1) {
            const int kbx = kin * p.a_box_elems;
            tma_load_2d_pair(smem + L.a_off + stage * L.a_bytes, &tmA, fb, term * p.term_stride + kbx, a_row, pol_a);
            tma_load_2d_pair(smem + L.b_off + stage * L.b_bytes, &tmB, fb, kbx, b_row, pol_b);
          } else {
            // k-blocks past this range's end are loaded (zeros past K) but not multiplied
            tma_load_3d_pair(smem + L.a_off + stage * L.a_bytes, &tmA, fb, a_row, term * p.term_kb + kin, pol_a);
            tma_load_3d_pair(smem + L.b_off + stage * L.b_bytes, &tmB, fb, b_row, kin, pol_b);
          }
          issued_mask |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (trace) {
        trace[2] = globaltimer();
        trace[8] = wait_empty;
      }
      if (*abort_flag && crank == 0) {
        // The even CTA's full barriers count both CTAs' copies: once they are
        // complete, no copy of either CTA is in flight.
        for (int s = 0; s < p.stages; ++s)
          if (issued_mask & (1u << s))
            mbar_wait(full_bar + s, (last_phase >> s) & 1u, nullptr, abort_flag, kDevTimeoutDrain, false);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (even CTA)
    if (lane == 0 && crank == 0) {
      pdl_wait_prior();
      const int T = (MODE == TcMode::kBf16Norm) ? active_terms(p) : 1;
      const uint32_t idesc = kInt ? umma_idesc(2, 1, kPairRows, p.bn) : umma_idesc(1, 1, kPairRows, p.bn);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      unsigned long long wait_accum = 0, wait_full = 0;  // trace: time waiting for TMEM / for stages
      int a_row, tn, kb0, kb1;
      for (int i = 0; ok && tile_of(i, a_row, tn, kb0, kb1); ++i) {
        const int buf = i & 1;
        const unsigned long long tw0 = trace ? globaltimer() : 0;
        if (!mbar_wait(tempty_bar + buf, ((i >> 1) & 1) ^ 1, p.err, abort_flag, kDevTimeoutAccumFree)) break;
        if (trace) wait_accum += globaltimer() - tw0;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * p.bn);
        const int nkb = kb1 - kb0;
        const int nops = (nkb + p.kps - 1) / p.kps;
        for (int j = 0; j < T * nops; ++j) {
          const unsigned long long tw1 = trace ? globaltimer() : 0;
          if (!mbar_wait(full_bar + stage, phase, p.err, abort_flag, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          if (trace) wait_full += globaltimer() - tw1;
          tc_fence_after();
          if (trace && !issued) trace[3] = globaltimer();
          const int o = j % nops;
          const int nv = min(p.kps, nkb - o * p.kps);  // k-blocks of this stage inside the range
          const uint32_t a_addr = smem_u32(smem + L.a_off + stage * L.a_bytes);
          const uint32_t b_addr = smem_u32(smem + L.b_off + stage * L.b_bytes);
          for (int v = 0; v < nv; ++v) {
            #pragma unroll
            for (uint32_t u = 0; u < 4; ++u) {
              const uint64_t ad = umma_desc_sw128(a_addr + v * a_kb_bytes + 32 * u);
              const uint64_t bd = umma_desc_sw128(b_addr + v * b_kb_bytes + 32 * u);
              const uint32_t acc = (j > 0 || v > 0 || u > 0) ? 1u : 0u;
              if constexpr (kInt)
                umma_i8_pair(d_tmem, ad, bd, idesc, acc);
              else
                umma_f16_pair(d_tmem, ad, bd, idesc, acc);
            }
          }
          issued = true;
          umma_commit_pair(empty_bar + stage);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar + buf);
      }
      if (trace) {
        trace[4] = globaltimer();
        trace[9] = wait_full;
        trace[10] = wait_accum;
      }
      if (issued && *abort_flag) {
        umma_commit_pair(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, abort_flag, kDevTimeoutDrain, false);
      }
    }
  } else {
    // ------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int ethread = threadIdx.x - 64;
    pdl_wait_prior();
    unsigned long long epi_wait = 0;  // trace: time waiting for accumulators
    unsigned long long epi_ld = 0, epi_fin = 0;  // trace: time in TMEM loads / finishing and storing
    int a_row, tn, kb0, kb1;
    for (int i = 0; tile_of(i, a_row, tn, kb0, kb1); ++i) {
      const int buf = i & 1;
      const int grow = a_row + row;
      float scale_n = 0.f;
      if constexpr (kSwap) {
        // the tile's per-token exponents and flags, and this row's scale
        named_bar_sync(1, kEpiThreads);
        if (ethread < p.tok_per_tile) {
          const int t = tn * p.tok_per_tile + ethread;
          s_exp[ethread] = t < p.n_tokens ? __ldg(p.exps + t) : 0;
          s_bad[ethread] = t < p.n_tokens ? __ldg(p.nonfinite + t) : 0;
        }
        if (grow < p.n_out) scale_n = __ldg(p.scale + grow);
        named_bar_sync(1, kEpiThreads);
      } else if constexpr (MODE == TcMode::kI8Norm) {
        // column scales of the tile, staged while the accumulator is computed
        named_bar_sync(1, kEpiThreads);
        if (p.out || p.npeers)
          for (int j = ethread; j < p.bn; j += kEpiThreads) {
            const int col = tn * p.bn + j;
            s_scale[j] = col < p.cols ? __ldg(p.scale + col) : 0.f;
          }
        named_bar_sync(1, kEpiThreads);
      }
      const unsigned long long tw = trace ? globaltimer() : 0;
      if (!mbar_wait(tfull_bar + buf, (i >> 1) & 1, p.err, abort_flag, kDevTimeoutAccum, false)) break;
      if (trace) epi_wait += globaltimer() - tw;
      tc_fence_after();
      if (trace && ethread == 0 && i == 0) trace[5] = globaltimer();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * p.bn;
      if constexpr (kSwap) {
        // 48 columns = 16 tokens per chunk
        const int nch = p.bn / 48;
        for (int ci = half; ci < nch; ci += 2) {
          const int c = ci * 48;
          uint32_t v[48];
          __syncwarp();
          const unsigned long long tl0 = trace ? globaltimer() : 0;
          tmem_ld16(tbase + c, *reinterpret_cast<uint32_t(*)[16]>(v));
          tmem_ld16(tbase + c + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
          tmem_ld16(tbase + c + 32, *reinterpret_cast<uint32_t(*)[16]>(v + 32));
          tmem_ld_wait();
          const unsigned long long tl1 = trace ? globaltimer() : 0;
          epi_swap48<MODE>(p, grow, tn * p.tok_per_tile, c / 3, scale_n, s_exp, s_bad, v);
          if (trace) {
            epi_ld += tl1 - tl0;
            epi_fin += globaltimer() - tl1;
          }
        }
      } else {
        const int nch = p.bn / 16;
        for (int ci = half; ci < nch; ci += 2) {
          const int c = ci * 16;
          uint32_t v[16];
          __syncwarp();
          tmem_ld16(tbase + c, v);
          tmem_ld_wait();
          epi_norm16<MODE>(p, grow - lane, tn * p.bn + c, v, s_stage, s_scale + c);
        }
      }
      // this warp has read the accumulator: the even CTA's MMA may reuse it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (crank == 0)
          mbar_arrive(tempty_bar + buf);
        else
          mbar_arrive_remote(tempty_even + buf * 8);
      }
    }
    if (trace && threadIdx.x == 64) {
      trace[6] = globaltimer();
      trace[11] = epi_wait;
      trace[12] = epi_ld;
      trace[13] = epi_fin;
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(done_bar);
  }

  if (warp == 1) {
    __syncwarp();
    mbar_wait(done_bar, 0, p.err, abort_flag, kDevTimeoutDrain, false);
    tc_fence_after();
  }
  // Neither CTA leaves (or releases TMEM) while the other may still arrive on
  // its barriers or run MMAs on its operands and accumulators.
  __syncwarp();
  cluster_arrive_release();
  cluster_wait_acquire();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, p.tmem_cols);
    if (trace && lane == 0) trace[7] = globaltimer();
  }
  // Row-sharded call: the same completion handshake as tc_gemm_kernel.
  if (p.npeers > 0 && warp >= 2) {
    fence_sc_sys();
    named_bar_sync(1, kEpiThreads);
    if (threadIdx.x == 64) {
      const unsigned done = static_cast<unsigned>(atom_add_acq_rel_gpu(p.done_ctr, 1u)) + 1u;
      if (done == gridDim.x) {
        *p.done_ctr = 0u;
        for (int q = 0; q < p.npeers; ++q) red_add_release_sys(p.peer_inbox[q], 1u);
        const unsigned* own = p.peer_inbox[p.rank];
        const unsigned long long t0 = globaltimer();
        while (static_cast<int>(ld_acquire_sys(own) - p.inbox_target) < 0) {
          if (globaltimer() - t0 > kPeerWaitLimitNs) {
            atomicCAS(p.err, 0, kDevTimeoutPeers);
            break;
          }
          __nanosleep(256);
        }
      }
    }
  }
}

}  // namespace vmlm
