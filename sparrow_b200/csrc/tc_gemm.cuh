// tc_gemm.cuh -- the tcgen05 GEMM used by every fast path of the library.
//
// One persistent, warp-specialised kernel computes D = A[rows,K] . B[cols,K]^T
// with both operands K-major in HBM, staged by TMA (128-byte swizzle, no
// multicast) through an mbarrier ring, multiplied by tcgen05.mma into a
// double-buffered TMEM accumulator, and finished by an epilogue that depends
// on the mode:
//
//   kQ8Swap    A = int8 weight rows W[n,:], B = int8 digit planes of the f32
//              activations (row 3t+p is plane p of token t). kind::i8, s32
//              accumulators. Epilogue recombines the three planes exactly in
//              int64, applies the token's power-of-two exponent and scale[n]:
//              C[t][n] = f32(f64(sum_p 256^p acc_p) * 2^-e_t) * scale[n].
//   kBf16Swap  A = bf16 weight rows, B = bf16 split terms of the f32
//              activations (row 3t+j is term j of token t). kind::f16 with f32
//              accumulators; the epilogue adds the three terms.
//   kBf16Norm  A = bf16 split terms of the activations laid out term-major
//              along K (K' = T*K, T read on the device), B = bf16 weight rows.
//              C[m][n] straight from the accumulator.
//   kI8Norm    A = int8 activations X[m,:], B = int8 weights W[n,:]:
//              C[m][n] = f32(acc) * scale[n], and/or the raw int32 acc.
//   kF32Norm   A and B = bf16 split terms of two f32 operands, both laid out
//              term-major along K; the passes run the term pairs (i, j) with
//              i + j <= 2. C[m][n] (+)= the f32 accumulator; outputs touching
//              a NaN/Inf row are recomputed exactly from the terms.
//
// Warp roles (320 threads): warp 0 issues TMA, warp 1 owns TMEM and issues
// the MMAs, warps 2..9 are the epilogue: warp w reads TMEM lanes
// 32*(w%4) .. +31 and finishes every other column chunk of them.
//
// Scheduling is static. Units are (tile, k-block) pairs ordered tile-major.
// Either every CTA takes whole tiles round-robin, or each CTA takes a
// contiguous range of units:
//   swap modes (stream-K): the CTA that brings a split tile's counter to the
//     full k-block count finishes it; contributors add one combined value per
//     token atomically into a self-clearing slot (exact for Q8; last-bit order
//     dependent for bf16);
//   normal modes (explicit K split over a thread-block cluster of csplit
//     CTAs): partial tiles are exchanged through distributed shared memory and
//     each CTA finishes a column slice, summing in rank order (deterministic).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "ptx.cuh"

namespace vmlm {

enum class TcMode : int { kQ8Swap = 0, kBf16Swap = 1, kBf16Norm = 2, kI8Norm = 3, kF32Norm = 4 };

constexpr int kTileRows = 128;        // UMMA M
constexpr int kBlockBytes = 128;      // bytes of K per stage (one 128B swizzle row)
constexpr int kThreads = 320;        // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpiWarps = 8;         // two per TMEM lane quarter, splitting the columns
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kMaxSmem = 227 * 1024;
constexpr int kMaxTokPerTile = 128;   // swap modes: tokens per column tile (bn/3 <= 85)
constexpr int kMaxPeers = 8;          // ranks of a row-sharded call

struct TcParams {
  int rows;          // extent of A rows (W rows in swap modes, tokens in normal modes)
  int cols;          // extent of B rows (plane/term rows in swap modes, W rows in normal modes)
  int bn;            // UMMA N per tile (multiple of 16, <= 256; multiple of 48 in swap modes)
  int kb_per_term;   // k-blocks per pass over K
  int max_terms;     // kBf16Norm / kF32Norm: terms allocated per operand (1..3); 1 otherwise
  int tiles_m, tiles_n;
  int streamk;       // 1 = stream-K ranges, 0 = round-robin whole tiles
  int tm_fastest;    // tile index -> (tm, tn): 1 = tm varies fastest, 0 = tn fastest
  int stages;
  int tmem_cols;     // allocated TMEM columns (power of two >= 2*bn)
  int a_box_elems;   // TMA box inner extent of A/B in elements (128 int8 or 64 bf16)
  int term_stride;   // kBf16Norm / kF32Norm: element offset between terms along K
  // epilogue
  float* out;        // C, row-major
  long long ldo;     // row stride of C (elements)
  int vec_out;       // C (and acc_out) rows are 16-byte aligned: vector stores allowed
  int32_t* acc_out;  // kI8Norm: optional raw accumulators (row stride ldo)
  const float* scale;
  const int* exps;        // kQ8Swap: per-token exponent e (value = v * 2^-e)
  const int* nonfinite;   // per-token flag: row of x holds NaN/Inf
  const int* term_flags;  // kBf16Norm / kF32Norm: OR over A's rows of (1<<j) for every non-zero term j
  int n_tokens;           // tokens (swap modes: real tokens; used for bounds)
  int tok_per_tile;       // swap modes: tokens per column tile (bn/3)
  int n_out;              // swap modes: W rows (bounds on n)
  // non-finite fallback (swap modes): exact f32 recompute of flagged tokens
  const float* x;
  long long ldx;
  const void* w;     // int8 or bf16 weight rows (row stride k)
  int k;
  // split-tile fixup
  uint32_t* slots;   // swap modes: [grid] slots of [tok][128] combined values, all zero between calls
  int* counters;     // [tiles] k-blocks finished so far (self-resetting)
  int csplit;        // normal modes: > 1 = each tile's K split over a cluster of csplit CTAs
  int ksplit;        // tc2_gemm_kernel, normal modes: K ranges per pair tile (1 or 2); with 2 each
                     // range's partial is added into C (zeroed beforehand) with red.global.add
  int kps;           // tc2_gemm_kernel: k-blocks per stage (1: 2-D tensor maps; 2..3: 3-D maps, one
                     // load per operand per stage; A's k-block coordinate of term t is t * term_kb + kb)
  int term_kb;       // k-blocks per term in A's 3-D map (kBf16Norm)
  // kF32Norm (C = A . B^T, both operands f32 split into three bf16 terms):
  // B's terms at j * term_stride along its K, B's OR word, per-row NaN/Inf
  // flags of A and B, both term buffers ([rows][3 * term_stride]) for the
  // exact recompute of outputs that touch a NaN/Inf row, and acc_c = add the
  // old C (C += A . B^T).
  const int* term_flags_b;
  const int* nf_a;
  const int* nf_b;
  const uint16_t* terms_a;
  const uint16_t* terms_b;
  int acc_c;
  // Row-sharded call with the all-gather in the epilogue (npeers > 0): this
  // rank computes output columns [col_off, col_off + its rows) and stores every
  // value into all npeers ranks' full C (peer_out[q], row stride ldo) over
  // NVLink. When its last CTA is done it adds 1 to every rank's inbox, and the
  // kernel ends once its own inbox reaches inbox_target (npeers per call made
  // on that inbox so far, this one included).
  int npeers;
  int rank;
  long long col_off;
  float* peer_out[kMaxPeers];
  unsigned* peer_inbox[kMaxPeers];
  unsigned* done_ctr;    // this rank's CTA completion counter (self-resetting)
  unsigned inbox_target;
  int* err;          // device error word
  unsigned long long* trace;  // optional: kTraceSlots globaltimer stamps per CTA (diagnostics)
};

// Trace slots (per CTA): [0] kernel start, [1] producer past the wait for the
// previous kernel, [2] producer done issuing, [3] first stage consumed by the
// MMA warp, [4] last accumulator committed, [5] first accumulator seen by the
// epilogue, [6] epilogue done, [7] TMEM released; then summed waits (ns):
// [8] producer for free stages, [9] MMA for loaded stages, [10] MMA for a free
// accumulator, [11] epilogue for a finished accumulator; epilogue phases (ns,
// summed): [12] split tiles: publishing partials / whole tiles: TMEM loads,
// [13] split tiles: counting arrivals / whole tiles: finishing and storing,
// [14] split tiles: finishing; [15] work items * 65536 + tiles finished.
constexpr int kTraceSlots = 16;

struct TcSmem {
  uint32_t a_off, b_off, bar_off, meta_off, stg_off;  // offsets from the 1024-aligned base
  uint32_t a_bytes, b_bytes, total;
};

__host__ __device__ inline TcSmem tc_smem_layout(int stages, int bn) {
  TcSmem s;
  s.a_bytes = kTileRows * kBlockBytes;
  s.b_bytes = static_cast<uint32_t>(bn) * kBlockBytes;
  s.a_off = 0;
  s.b_off = s.a_off + stages * s.a_bytes;
  s.bar_off = s.b_off + stages * s.b_bytes;
  // full[stages], empty[stages], tmem_full[2], tmem_empty[2], drain, done, then 64 bytes of words
  s.meta_off = s.bar_off + (2 * stages + 6) * 8 + 64;
  // per-tile token table: exps[kMaxTokPerTile], nonfinite[kMaxTokPerTile]
  s.stg_off = s.meta_off + 2 * kMaxTokPerTile * 4;
  // per-epilogue-warp store staging (32 rows x 17 words); +1024 for base alignment
  s.total = s.stg_off + kEpiWarps * 32 * 17 * 4 + 1024;
  return s;
}

struct WorkItem {
  int tile, kb0, kb1;  // k-blocks [kb0, kb1) of the tile (in units of the tile's KB)
  bool partial;
};

// Static schedule over (tile, k-block) units of one term pass.
struct Sched {
  long long units;  // total units
  int kb_tile;      // k-blocks per tile
  int tiles;
  int grid;
  int streamk;

  __device__ __forceinline__ long long start(int c) const { return (static_cast<long long>(c) * units) / grid; }

  // i-th work item of CTA c; returns false when exhausted.
  __device__ __forceinline__ bool item(int c, int i, long long& cursor, WorkItem& w) const {
    if (!streamk) {
      long long t = static_cast<long long>(c) + static_cast<long long>(i) * grid;
      if (t >= tiles) return false;
      w.tile = static_cast<int>(t);
      w.kb0 = 0;
      w.kb1 = kb_tile;
      w.partial = false;
      return true;
    }
    const long long end = start(c + 1);
    if (i == 0) cursor = start(c);
    if (cursor >= end) return false;
    const long long tile = cursor / kb_tile;
    const int kb0 = static_cast<int>(cursor - tile * kb_tile);
    long long kb1 = kb0 + (end - cursor);
    if (kb1 > kb_tile) kb1 = kb_tile;
    w.tile = static_cast<int>(tile);
    w.kb0 = kb0;
    w.kb1 = static_cast<int>(kb1);
    w.partial = !(kb0 == 0 && kb1 == kb_tile);
    cursor += kb1 - kb0;
    return true;
  }

  // CTA that owns unit u: the largest c with start(c) <= u (every range is
  // non-empty because the host launches at most `units` CTAs).
  __device__ __forceinline__ int owner(long long u) const {
    long long c = (u * grid) / units;
    if (c > grid - 1) c = grid - 1;
    while (c > 0 && start(static_cast<int>(c)) > u) --c;
    while (c + 1 < grid && start(static_cast<int>(c + 1)) <= u) ++c;
    return static_cast<int>(c);
  }
};

// Number of split terms with any non-zero value (term_flags points at the OR of
// all tokens' flags, written by the prep kernel).
__device__ __forceinline__ int terms_of_word(const int* word, int max_terms) {
  if (max_terms <= 1) return 1;
  const int orv = __ldcg(word);
  int T = 1;
  if (orv & 2) T = 2;
  if (orv & 4) T = 3;
  return T < max_terms ? T : max_terms;
}

__device__ __forceinline__ int active_terms(const TcParams& p) { return terms_of_word(p.term_flags, p.max_terms); }

// The passes over K: a list of (A term i, B term j) pairs, 4 bits each
// (i | j << 2) in pass order; *np = their count. kBf16Norm runs A's active
// terms against the bf16 weights; kF32Norm the pairs with i + j <= 2 of both
// operands' active terms (the dropped products are below 2^-24 relative),
// smallest first: the tensor cores' f32 accumulation does not round each add
// to nearest, so the correction passes accumulate while the accumulator is
// still small, and the hi x hi pass comes last.
template <TcMode MODE>
__device__ __forceinline__ uint32_t term_pairs(const TcParams& p, int* np) {
  if constexpr (MODE == TcMode::kBf16Norm) {
    const int T = active_terms(p);
    *np = T;
    return 0x210u & ((1u << (4 * T)) - 1u);
  } else if constexpr (MODE == TcMode::kF32Norm) {
    const int ta = active_terms(p), tb = terms_of_word(p.term_flags_b, p.max_terms);
    constexpr uint32_t kCand = 0x041852u;  // (2,0) (1,1) (0,2) (1,0) (0,1) (0,0)
    uint32_t list = 0;
    int n = 0;
    #pragma unroll
    for (int c = 0; c < 6; ++c) {
      const uint32_t code = (kCand >> (4 * c)) & 15u;
      if (static_cast<int>(code & 3u) < ta && static_cast<int>(code >> 2) < tb) {
        list |= code << (4 * n);
        ++n;
      }
    }
    *np = n;
    return list;
  } else {
    *np = 1;
    return 0u;
  }
}

// ------------------------------------------------------------- epilogues

// Store a 32-row x 16-column block held one row per lane (lane = row - row0)
// through a per-warp shared buffer, so that each store instruction writes 8
// rows x 64 contiguous bytes instead of 32 rows x 16 bytes.
// kAdd: f32 values added to the destination's old values (C += ...).
// kRed: f32 values added to the destination in L2 (red.global.add), for
// partial sums of one output from two CTAs; f32 addition is commutative, so
// two partials added into a zeroed C give the same bits in either order.
template <bool kAdd = false, bool kRed = false>
__device__ __forceinline__ void store_block_32x16(uint32_t* dst, long long ld, int row0, int nrows, int col0,
                                                  int ncols, bool vec, uint32_t* buf, const uint32_t (&v)[16]) {
  const int lane = threadIdx.x & 31;
  #pragma unroll
  for (int j = 0; j < 16; ++j) buf[lane * 17 + j] = v[j];
  __syncwarp();
  #pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2);
    const int c = (lane & 3) * 4;
    const int grow = row0 + r;
    if (grow < nrows) {
      uint32_t* d = dst + static_cast<long long>(grow) * ld + col0 + c;
      const uint32_t* s = buf + r * 17 + c;
      if (vec && col0 + c + 4 <= ncols) {
        uint4 o = make_uint4(s[0], s[1], s[2], s[3]);
        if constexpr (kRed) {
          red_add_v4_f32(reinterpret_cast<float*>(d), o);
          continue;
        }
        if constexpr (kAdd) {
          const float4 q = *reinterpret_cast<const float4*>(d);
          o = make_uint4(__float_as_uint(__fadd_rn(__uint_as_float(o.x), q.x)),
                         __float_as_uint(__fadd_rn(__uint_as_float(o.y), q.y)),
                         __float_as_uint(__fadd_rn(__uint_as_float(o.z), q.z)),
                         __float_as_uint(__fadd_rn(__uint_as_float(o.w), q.w)));
        }
        *reinterpret_cast<uint4*>(d) = o;
      } else {
        for (int j = 0; j < 4; ++j)
          if (col0 + c + j < ncols) {
            if constexpr (kRed)
              red_add_f32(reinterpret_cast<float*>(d + j), __uint_as_float(s[j]));
            else if constexpr (kAdd)
              d[j] = __float_as_uint(__fadd_rn(__uint_as_float(s[j]), __uint_as_float(d[j])));
            else
              d[j] = s[j];
          }
      }
    }
  }
  __syncwarp();
}

// The K-split (csplit) epilogue of kBf16Norm, out of line so that one copy of
// the code serves the real calls and a dry run the epilogue warps make while
// the MMAs still run: code a warp executes for the first time waits for
// instruction fetches from L2 (about 2000 cycles per phase here), and the dry
// run takes those off the critical path.
//
// Publish 16 accumulator columns at TMEM address taddr: word j of each lane
// goes to cluster shared-memory address dst + j * stride.
__device__ __noinline__ void csplit_publish16(uint32_t taddr, uint32_t dst, uint32_t stride) {
  uint32_t v[16];
  tmem_ld16(taddr, v);
  tmem_ld_wait();
  #pragma unroll
  for (int j = 0; j < 16; ++j) st_cluster_u32(dst + static_cast<uint32_t>(j) * stride, v[j]);
}

// Finish 16 columns: this CTA's partial (TMEM at taddr) and the other S - 1
// partials in shared memory (sender slot s at recv + s * slot_stride, column j
// at j * col_stride), summed in rank order in f32, stored as a 32 x 16 block
// of C (store_block_32x16's arguments; nrows = 0 stores nothing).
__device__ __noinline__ void csplit_finish16_f32(uint32_t taddr, const uint32_t* recv, int slot_stride,
                                                 int col_stride, int S, int rank, uint32_t* dst, long long ld,
                                                 int row0, int nrows, int col0, int ncols, int vec, uint32_t* buf) {
  uint32_t own[16], v[16];
  tmem_ld16(taddr, own);
  tmem_ld_wait();
  #pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = 0u;
  for (int q = 0; q < S; ++q) {
    const uint32_t* src = recv + (q - (q > rank ? 1 : 0)) * slot_stride;
    #pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t a = (q == rank) ? own[j] : src[j * col_stride];
      v[j] = __float_as_uint(__fadd_rn(__uint_as_float(v[j]), __uint_as_float(a)));
    }
  }
  store_block_32x16(dst, ld, row0, nrows, col0, ncols, vec != 0, buf, v);
}

// Exact f32 recompute of C[t][n] for the f32 GEMM when row t of A or row n of
// B holds NaN / Inf: the values are rebuilt from their three terms (exact, and
// NaN / Inf survive in the first term) and summed sequentially. Out of line
// (a cold path).
__device__ __noinline__ float f32_terms_dot(const uint16_t* ta, const uint16_t* tb, int k, int kp) {
  auto val = [&](const uint16_t* t, int kk) {
    const float h = __uint_as_float(static_cast<uint32_t>(t[kk]) << 16);
    const float m = __uint_as_float(static_cast<uint32_t>(t[kp + kk]) << 16);
    const float l = __uint_as_float(static_cast<uint32_t>(t[2 * kp + kk]) << 16);
    return __fadd_rn(__fadd_rn(h, m), l);
  };
  float s = 0.f;
  for (int kk = 0; kk < k; ++kk) s = __fadd_rn(s, __fmul_rn(val(ta, kk), val(tb, kk)));
  return s;
}

// Finish 16 columns [col0, col0+16) of the warp's 32 accumulator rows
// (row0 = first row of the warp) in a normal mode. s_scale points at the
// chunk's 16 column scales in shared memory (kI8Norm).
template <TcMode MODE>
__device__ __forceinline__ void epi_norm16(const TcParams& p, int row0, int col0, const uint32_t (&v)[16],
                                           uint32_t* buf, const float* s_scale) {
  if constexpr (MODE == TcMode::kI8Norm) {
    if (p.acc_out)
      store_block_32x16(reinterpret_cast<uint32_t*>(p.acc_out), p.ldo, row0, p.rows, col0, p.cols, p.vec_out, buf,
                        v);
    if (p.out || p.npeers) {
      uint32_t f[16];
      #pragma unroll
      for (int j = 0; j < 16; ++j)
        f[j] = __float_as_uint(__fmul_rn(__int2float_rn(static_cast<int>(v[j])), s_scale[j]));
      if (p.npeers == 0) {
        store_block_32x16(reinterpret_cast<uint32_t*>(p.out), p.ldo, row0, p.rows, col0, p.cols, p.vec_out, buf, f);
      } else {
        for (int q = 0; q < p.npeers; ++q)
          store_block_32x16(reinterpret_cast<uint32_t*>(p.peer_out[q] + p.col_off), p.ldo, row0, p.rows, col0,
                            p.cols, p.vec_out, buf, f);
      }
    }
  } else if constexpr (MODE == TcMode::kF32Norm) {
    uint32_t f[16];
    #pragma unroll
    for (int j = 0; j < 16; ++j) f[j] = v[j];
    if ((__ldcg(p.term_flags) | __ldcg(p.term_flags_b)) & 256) {
      // some row of A or B holds NaN / Inf: recompute the outputs that touch one
      const int t = row0 + (threadIdx.x & 31);
      const bool bad_t = t < p.rows && __ldg(p.nf_a + t);
      const long long tp = 3ll * p.term_stride;
      for (int j = 0; j < 16; ++j) {
        const int n = col0 + j;
        if (t < p.rows && n < p.cols && (bad_t || __ldg(p.nf_b + n)))
          f[j] = __float_as_uint(f32_terms_dot(p.terms_a + t * tp, p.terms_b + n * tp, p.k, p.term_stride));
      }
    }
    if (p.acc_c)
      store_block_32x16<true>(reinterpret_cast<uint32_t*>(p.out), p.ldo, row0, p.rows, col0, p.cols, p.vec_out, buf,
                              f);
    else
      store_block_32x16(reinterpret_cast<uint32_t*>(p.out), p.ldo, row0, p.rows, col0, p.cols, p.vec_out, buf, f);
  } else if (p.npeers == 0) {
    if (MODE == TcMode::kBf16Norm && p.ksplit > 1)
      store_block_32x16<false, true>(reinterpret_cast<uint32_t*>(p.out), p.ldo, row0, p.rows, col0, p.cols, p.vec_out,
                                     buf, v);
    else
      store_block_32x16(reinterpret_cast<uint32_t*>(p.out), p.ldo, row0, p.rows, col0, p.cols, p.vec_out, buf, v);
  } else {
    for (int q = 0; q < p.npeers; ++q)
      store_block_32x16(reinterpret_cast<uint32_t*>(p.peer_out[q] + p.col_off), p.ldo, row0, p.rows, col0, p.cols,
                        p.vec_out, buf, v);
  }
}

// Exact f32 recompute of one output for a token whose activations hold NaN or
// Inf (the digit-plane / split-term encodings cannot carry them). Summation is
// sequential, which gives the same NaN/Inf classification as any order.
// Cold paths of the epilogue stay out of line (plain arguments, no parameter
// struct), so the unrolled hot loops that call them stay small in the
// instruction cache.
__device__ __noinline__ float nonfinite_dot_q8(const float* xr, const int8_t* wr, int k, float sc) {
  float s = 0.f;
  for (int kk = 0; kk < k; ++kk) s = __fadd_rn(s, __fmul_rn(xr[kk], static_cast<float>(wr[kk])));
  return __fmul_rn(s, sc);
}

__device__ __noinline__ float nonfinite_dot_bf16(const float* xr, const uint16_t* wr, int k) {
  float s = 0.f;
  for (int kk = 0; kk < k; ++kk)
    s = __fadd_rn(s, __fmul_rn(xr[kk], __uint_as_float(static_cast<uint32_t>(wr[kk]) << 16)));
  return s;
}

// f32(v * 2^-e) * sc for exponents outside the single-precision fast path.
__device__ __noinline__ float q8_scale_wide(long long v, int e, float sc) {
  return __fmul_rn(__double2float_rn(ldexp(static_cast<double>(v), -e)), sc);
}

template <TcMode MODE>
__device__ __forceinline__ float nonfinite_dot(const TcParams& p, int t, int n) {
  const float* xr = p.x + static_cast<long long>(t) * p.ldx;
  if constexpr (MODE == TcMode::kQ8Swap)
    return nonfinite_dot_q8(xr, static_cast<const int8_t*>(p.w) + static_cast<long long>(n) * p.k, p.k,
                            __ldg(p.scale + n));
  else
    return nonfinite_dot_bf16(xr, static_cast<const uint16_t*>(p.w) + static_cast<long long>(n) * p.k, p.k);
}

// Swap modes combine one token's three accumulator columns (token-major
// triples) into one value: the exact int64 digit-plane sum for Q8, the f32 sum
// of the three split terms for bf16. Split tiles reduce these combined values.
template <TcMode MODE>
struct SwapVal {
  using T = typename std::conditional<MODE == TcMode::kQ8Swap, unsigned long long, float>::type;
};

template <TcMode MODE>
__device__ __forceinline__ typename SwapVal<MODE>::T swap_combine(const uint32_t* v3) {
  if constexpr (MODE == TcMode::kQ8Swap) {
    const long long a0 = static_cast<int>(v3[0]);
    const long long a1 = static_cast<int>(v3[1]);
    const long long a2 = static_cast<int>(v3[2]);
    return static_cast<unsigned long long>(a2 * 65536ll + a1 * 256ll + a0);
  } else {
    return __fadd_rn(__uint_as_float(v3[0]), __fadd_rn(__uint_as_float(v3[1]), __uint_as_float(v3[2])));
  }
}

// Final value of output (t, n) from a token's combined accumulator. Q8:
// C = f32(v * 2^-e) * scale[n]. When v * 2^-e is a normal float (|e| in the
// checked range, v an integer), rounding v to f32 and then scaling by the exact
// power of two gives the same bits as the f64 route used otherwise.
template <TcMode MODE>
__device__ __forceinline__ void swap_finish(const TcParams& p, int n, int t, int lt, typename SwapVal<MODE>::T val,
                                            float sc, const int* s_exp, const int* s_bad) {
  float r;
  if (s_bad[lt]) {
    r = nonfinite_dot<MODE>(p, t, n);
  } else if constexpr (MODE == TcMode::kQ8Swap) {
    const long long v = static_cast<long long>(val);
    const int e = s_exp[lt];
    if (e >= -70 && e <= 100) {
      r = __fmul_rn(__fmul_rn(__ll2float_rn(v), __int_as_float((127 - e) << 23)), sc);
    } else {
      r = q8_scale_wide(v, e, sc);
    }
  } else {
    r = val;
  }
  const long long idx = static_cast<long long>(t) * p.ldo + n;
  if (p.npeers == 0) {
    p.out[idx] = r;
  } else {
    for (int q = 0; q < p.npeers; ++q) p.peer_out[q][idx + p.col_off] = r;
  }
}

// Finish 16 tokens (48 accumulator columns) of one weight row of a whole tile.
// lt0 is the chunk's first token within the tile, tok0 the tile's first token.
template <TcMode MODE>
__device__ __forceinline__ void epi_swap48(const TcParams& p, int n, int tok0, int lt0, float sc, const int* s_exp,
                                           const int* s_bad, const uint32_t (&v)[48]) {
  if (n >= p.n_out) return;
  #pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int lt = lt0 + j;
    const int t = tok0 + lt;
    if (t < p.n_tokens) swap_finish<MODE>(p, n, t, lt, swap_combine<MODE>(v + 3 * j), sc, s_exp, s_bad);
  }
}

// Add 16 accumulator values into a fixup slot (integer or f32 atomics; the
// return values are unused, so these compile to reductions).
template <bool kInt>
__device__ __forceinline__ void slot_add16(uint32_t* s, const uint32_t (&v)[16]) {
  // column-major slot: consecutive columns are kTileRows words apart
  #pragma unroll
  for (int j = 0; j < 16; ++j) {
    if constexpr (kInt)
      atomicAdd(reinterpret_cast<int*>(s + j * kTileRows), static_cast<int>(v[j]));
    else
      atomicAdd(reinterpret_cast<float*>(s + j * kTileRows), __uint_as_float(v[j]));
  }
}

// --------------------------------------------------------------- kernel

template <TcMode MODE>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const TcParams p) {
  constexpr bool kSwap = (MODE == TcMode::kQ8Swap || MODE == TcMode::kBf16Swap);
  constexpr bool kInt = (MODE == TcMode::kQ8Swap || MODE == TcMode::kI8Norm);
  constexpr uint32_t kMmaPerBlock = 4;  // 128 bytes of K / 32 bytes per UMMA
  const uint32_t idesc = kInt ? umma_idesc(2, 1, kTileRows, p.bn) : umma_idesc(1, 1, kTileRows, p.bn);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  const TcSmem L = tc_smem_layout(p.stages, p.bn);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty_bar = full_bar + p.stages;
  uint64_t* tfull_bar = empty_bar + p.stages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* done_bar = drain_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* bcast = reinterpret_cast<volatile int*>(tmem_slot + 2);
  int* s_exp = reinterpret_cast<int*>(smem + L.meta_off);
  int* s_bad = s_exp + kMaxTokPerTile;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
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
      mbar_init(tempty_bar + b, kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    mbar_init(done_bar, kEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // The next kernel in the stream may be scheduled now: kernels this library
  // launches as programmatic dependents wait for this one to complete before
  // they touch memory it reads or writes (they only prefetch weights first).
  pdl_launch_dependents();
  const uint32_t tmem_base = *tmem_slot;

  const int cta = blockIdx.x;
  // Units are k-blocks of one term pass; a kBf16Norm work item runs its
  // k-block range once per active term, so the schedule does not depend on
  // the term count that the previous kernel produces.
  auto make_sched = [&]() {
    Sched s;
    s.kb_tile = p.kb_per_term;
    s.tiles = p.tiles_m * p.tiles_n;
    s.units = static_cast<long long>(s.tiles) * s.kb_tile;
    s.grid = gridDim.x;
    s.streamk = p.streamk;
    return s;
  };
  // The weights (A in swap modes, B in normal modes) do not depend on the
  // previous kernel in the stream; the activations do. The producer issues the
  // weight half of its first stages before waiting for that kernel, so the
  // weight stream overlaps the activation preparation.
  constexpr bool kWeightIsA = kSwap;
  unsigned long long epi_wait = 0;  // trace: epilogue time waiting for accumulators
  unsigned long long epi_pub = 0, epi_cnt = 0, epi_fin = 0, epi_items = 0;  // trace: split-tile phases
  bool epi_cluster_done = false;  // csplit: this epilogue thread took both cluster barrier steps

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_a = kSwap ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = kSwap ? policy_evict_last() : policy_evict_first();
      int npre = 0;  // stages of item 0 whose weight half is already in flight
      uint32_t issued_mask0 = 0;
      const Sched sc = make_sched();
      if constexpr (MODE != TcMode::kF32Norm) {
        // The first k-blocks of item 0 belong to term 0 whatever T turns out to
        // be. (kF32Norm: both operands come from the previous kernel.)
        long long cur0 = 0;
        WorkItem w0;
        if (sc.item(cta, 0, cur0, w0)) {
          const int tm0 = p.tm_fastest ? w0.tile % p.tiles_m : w0.tile / p.tiles_n;
          const int tn0 = p.tm_fastest ? w0.tile / p.tiles_m : w0.tile % p.tiles_n;
          npre = min(p.stages, w0.kb1 - w0.kb0);
          issued_mask0 = npre >= 32 ? 0xffffffffu : ((1u << npre) - 1u);
          for (int s = 0; s < npre; ++s) {
            const int kx = (w0.kb0 + s) * p.a_box_elems;
            mbar_arrive_expect_tx(full_bar + s, L.a_bytes + L.b_bytes);
            if (kWeightIsA)
              tma_load_2d(smem + L.a_off + s * L.a_bytes, &tmA, full_bar + s, kx, tm0 * kTileRows, pol_a);
            else
              tma_load_2d(smem + L.b_off + s * L.b_bytes, &tmB, full_bar + s, kx, tn0 * p.bn, pol_b);
          }
        }
      }
      pdl_wait_prior();
      if (trace) trace[1] = globaltimer();
      int T;  // passes over K (term pairs)
      const uint32_t pairs = term_pairs<MODE>(p, &T);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = issued_mask0, last_phase = 0;  // per stage: ever issued / parity of last issue
      unsigned long long wait_empty = 0;         // trace: time waiting for free stages
      long long cur = 0;
      WorkItem w;
      bool ok = true;
      for (int i = 0; ok && sc.item(cta, i, cur, w); ++i) {
        const int tm = p.tm_fastest ? w.tile % p.tiles_m : w.tile / p.tiles_n;
        const int tn = p.tm_fastest ? w.tile / p.tiles_m : w.tile % p.tiles_n;
        const int nkb = w.kb1 - w.kb0;
        for (int j = 0; j < T * nkb; ++j) {
          const int pass = j / nkb;
          const uint32_t code = (pairs >> (4 * pass)) & 15u;  // A term | B term << 2
          const int kin = w.kb0 + (j - pass * nkb);
          const bool pre = (i == 0 && j < npre);
          const unsigned long long tw = trace ? globaltimer() : 0;
          if (!pre && !mbar_wait(empty_bar + stage, phase ^ 1, p.err, abort_flag, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (trace) wait_empty += globaltimer() - tw;
          uint8_t* sa = smem + L.a_off + stage * L.a_bytes;
          uint8_t* sb = smem + L.b_off + stage * L.b_bytes;
          if (!pre) mbar_arrive_expect_tx(full_bar + stage, L.a_bytes + L.b_bytes);
          const int kbx = kin * p.a_box_elems;
          const int ka = static_cast<int>(code & 3u) * p.term_stride + kbx;
          const int kb = static_cast<int>(code >> 2) * p.term_stride + kbx;
          if (!pre || !kWeightIsA) tma_load_2d(sa, &tmA, full_bar + stage, ka, tm * kTileRows, pol_a);
          if (!pre || kWeightIsA) tma_load_2d(sb, &tmB, full_bar + stage, kb, tn * p.bn, pol_b);
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
      if (*abort_flag) {
        // Copies already issued must land before this CTA's shared memory is released.
        for (int s = 0; s < p.stages; ++s)
          if (issued_mask & (1u << s))
            mbar_wait(full_bar + s, (last_phase >> s) & 1u, nullptr, abort_flag, kDevTimeoutDrain, false);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      pdl_wait_prior();
      const Sched sc = make_sched();
      int T;  // passes over K (term pairs)
      term_pairs<MODE>(p, &T);
      int stage = 0;
      uint32_t phase = 0;
      long long cur = 0;
      WorkItem w;
      bool ok = true;
      bool issued = false;
      unsigned long long wait_accum = 0, wait_full = 0;  // trace: time waiting for TMEM / for stages
      for (int i = 0; ok && sc.item(cta, i, cur, w); ++i) {
        const int buf = i & 1;
        const unsigned long long tw0 = trace ? globaltimer() : 0;
        if (!mbar_wait(tempty_bar + buf, ((i >> 1) & 1) ^ 1, p.err, abort_flag, kDevTimeoutAccumFree)) break;
        if (trace) wait_accum += globaltimer() - tw0;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * p.bn);
        const int nblk = T * (w.kb1 - w.kb0);
        for (int j = 0; j < nblk; ++j) {
          const unsigned long long tw1 = trace ? globaltimer() : 0;
          if (!mbar_wait(full_bar + stage, phase, p.err, abort_flag, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          if (trace) wait_full += globaltimer() - tw1;
          tc_fence_after();
          if (trace && !issued) trace[3] = globaltimer();
          const uint32_t a_addr = smem_u32(smem + L.a_off + stage * L.a_bytes);
          const uint32_t b_addr = smem_u32(smem + L.b_off + stage * L.b_bytes);
          #pragma unroll
          for (uint32_t u = 0; u < kMmaPerBlock; ++u) {
            const uint64_t ad = umma_desc_sw128(a_addr + 32 * u);
            const uint64_t bd = umma_desc_sw128(b_addr + 32 * u);
            const uint32_t acc = (j > 0 || u > 0) ? 1u : 0u;
            if constexpr (kInt)
              umma_i8(d_tmem, ad, bd, idesc, acc);
            else
              umma_f16(d_tmem, ad, bd, idesc, acc);
          }
          issued = true;
          umma_commit(empty_bar + stage);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar + buf);
      }
      if (trace) {
        trace[4] = globaltimer();
        trace[9] = wait_full;
        trace[10] = wait_accum;
      }
      if (issued && *abort_flag) {
        // Let in-flight MMAs finish before TMEM is released.
        umma_commit(drain_bar);
        mbar_wait(drain_bar, 0, nullptr, abort_flag, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;          // TMEM lanes 32*quarter .. +31
    const int half = (warp - 2) >> 2;      // which alternate column chunks this warp finishes
    const int row = quarter * 32 + lane;   // accumulator row within the tile
    const int ethread = threadIdx.x - 64;  // 0..kEpiThreads-1
    // Column chunks: 48 columns (16 tokens) in swap modes, 16 otherwise; warp
    // pair (quarter, half) takes chunks ci with ci % 2 == half.
    constexpr int kChunk = kSwap ? 48 : 16;
    if constexpr (MODE == TcMode::kBf16Norm) {
      if (p.csplit > 1) {
        // Dry run of the split-tile epilogue (see csplit_publish16): TMEM of
        // the idle second accumulator buffer (one item per CTA here), into
        // this warp's own staging buffer, and no stores to C.
        const uint32_t idle = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + p.bn;
        __syncwarp();
        csplit_publish16(idle, mapa_shared(smem_u32(s_stage) + lane * 4, cluster_ctarank()), 4);
        __syncwarp();
        csplit_finish16_f32(idle, s_stage, 0, 1, p.csplit, 0, reinterpret_cast<uint32_t*>(p.out), p.ldo, 0, 0, 0,
                            p.cols, 0, s_stage);
        __syncwarp();
      }
    }
    pdl_wait_prior();
    const Sched sc = make_sched();
    long long cur = 0;
    WorkItem w;
    for (int i = 0; sc.item(cta, i, cur, w); ++i) {
      const int buf = i & 1;
      const int tm = p.tm_fastest ? w.tile % p.tiles_m : w.tile / p.tiles_n;
      const int tn = p.tm_fastest ? w.tile / p.tiles_m : w.tile % p.tiles_n;
      const int grow = tm * kTileRows + row;  // A row (W row in swap modes, token in normal modes)
      const int tok0 = tn * p.tok_per_tile;
      float scale_n = 0.f;
      if constexpr (kSwap) {
        // Stage the tile's per-token metadata once (one load per thread) while
        // the accumulator is still being computed.
        named_bar_sync(1, kEpiThreads);
        if (ethread < p.tok_per_tile) {
          const int t = tok0 + ethread;
          s_exp[ethread] = (MODE == TcMode::kQ8Swap && t < p.n_tokens) ? __ldg(p.exps + t) : 0;
          s_bad[ethread] = (t < p.n_tokens) ? __ldg(p.nonfinite + t) : 0;
        }
        if (MODE == TcMode::kQ8Swap && grow < p.n_out) scale_n = __ldg(p.scale + grow);
        named_bar_sync(1, kEpiThreads);
      } else if constexpr (MODE == TcMode::kI8Norm) {
        // Stage the tile's column scales (bn <= 256 floats, in the token-table
        // words) while the accumulator is still being computed.
        named_bar_sync(1, kEpiThreads);
        if (p.out || p.npeers) {
          float* s_scale = reinterpret_cast<float*>(s_exp);
          for (int j = ethread; j < p.bn; j += kEpiThreads) {
            const int col = tn * p.bn + j;
            s_scale[j] = col < p.cols ? __ldg(p.scale + col) : 0.f;
          }
        }
        named_bar_sync(1, kEpiThreads);
      }
      const unsigned long long tw = trace ? globaltimer() : 0;
      if (!mbar_wait(tfull_bar + buf, (i >> 1) & 1, p.err, abort_flag, kDevTimeoutAccum, false)) break;
      if (trace) epi_wait += globaltimer() - tw;
      tc_fence_after();
      if (trace && ethread == 0 && i == 0) trace[5] = globaltimer();
      if (trace) epi_items += 65536;
      const unsigned long long tp0 = trace ? globaltimer() : 0;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * p.bn;
      const int nch = p.bn / kChunk;
      // last chunk of this warp (largest ci < nch with ci % 2 == half), -1 if none
      const int my_last = (nch - 1 - half) < 0 ? -1 : (nch - 1) - (((nch - 1) ^ half) & 1);
      // this warp has read all its TMEM columns: let the MMA warp reuse the buffer
      auto release_accum = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar + buf);
      };

      if (!w.partial) {
        if (my_last < 0) release_accum();
        if constexpr (kSwap) {
          for (int ci = half; ci < nch; ci += 2) {
            const int c = ci * kChunk;
            uint32_t v[48];
            __syncwarp();
            const unsigned long long tl0 = trace ? globaltimer() : 0;
            tmem_ld16(tbase + c, *reinterpret_cast<uint32_t(*)[16]>(v));
            tmem_ld16(tbase + c + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
            tmem_ld16(tbase + c + 32, *reinterpret_cast<uint32_t(*)[16]>(v + 32));
            tmem_ld_wait();
            const unsigned long long tl1 = trace ? globaltimer() : 0;
            if (ci == my_last) release_accum();
            epi_swap48<MODE>(p, grow, tok0, c / 3, scale_n, s_exp, s_bad, v);
            if (trace) {
              epi_pub += tl1 - tl0;
              epi_cnt += globaltimer() - tl1;
            }
          }
        } else {
          for (int ci = half; ci < nch; ci += 2) {
            const int c = ci * kChunk;
            uint32_t v[16];
            __syncwarp();
            const unsigned long long tl0 = trace ? globaltimer() : 0;
            tmem_ld16(tbase + c, v);
            tmem_ld_wait();
            const unsigned long long tl1 = trace ? globaltimer() : 0;
            if (ci == my_last) release_accum();
            epi_norm16<MODE>(p, grow - lane, tn * p.bn + c, v, s_stage, reinterpret_cast<const float*>(s_exp) + c);
            if (trace) {
              epi_pub += tl1 - tl0;              // whole tiles: time in TMEM loads
              epi_cnt += globaltimer() - tl1;    // whole tiles: time finishing and storing
            }
          }
        }
        continue;
      }

      if constexpr (!kSwap) {
        if (p.csplit > 1) {
          // K split over a cluster of S CTAs (one item each). CTA `rank`
          // finishes columns [rank*slice, (rank+1)*slice) of the tile: the
          // others send it their partials of those columns through
          // distributed shared memory, into its stage buffers, which are idle
          // once every CTA of the cluster has finished its MMAs. Received
          // partials are [sender slot][column][128 rows] 32-bit words; the sum
          // runs in rank order, so f32 results do not depend on timing.
          const int S = p.csplit;
          const int rank = static_cast<int>(cluster_ctarank());
          const int slice = p.bn / S;
          const int nsc = slice / 16;
          const uint32_t* recv = reinterpret_cast<const uint32_t*>(smem);
          cluster_arrive_release();
          cluster_wait_acquire();  // A: every CTA of the cluster is past its MMAs
          for (int q = 0; q < S; ++q) {
            if (q == rank) continue;
            const uint32_t base = mapa_shared(smem_u32(smem), static_cast<uint32_t>(q)) +
                                  static_cast<uint32_t>(((rank - (rank > q ? 1 : 0)) * slice * kTileRows + row) * 4);
            for (int ci = half; ci < nsc; ci += 2) {
              __syncwarp();
              if constexpr (MODE == TcMode::kBf16Norm) {
                csplit_publish16(tbase + q * slice + ci * 16, base + static_cast<uint32_t>(ci * 16 * kTileRows * 4),
                                 kTileRows * 4);
              } else {
                uint32_t v[16];
                tmem_ld16(tbase + q * slice + ci * 16, v);
                tmem_ld_wait();
                #pragma unroll
                for (int j = 0; j < 16; ++j)
                  st_cluster_u32(base + static_cast<uint32_t>((ci * 16 + j) * kTileRows * 4), v[j]);
              }
            }
          }
          const unsigned long long tp1 = trace ? globaltimer() : 0;
          if (trace) epi_pub += tp1 - tp0;
          cluster_arrive_release();
          cluster_wait_acquire();  // B: all partials delivered
          const unsigned long long tp2 = trace ? globaltimer() : 0;
          if (trace) epi_cnt += tp2 - tp1;
          for (int ci = half; ci < nsc; ci += 2) {
            if constexpr (MODE == TcMode::kBf16Norm) {
              __syncwarp();
              csplit_finish16_f32(tbase + rank * slice + ci * 16, recv + ci * 16 * kTileRows + row, slice * kTileRows,
                                  kTileRows, S, rank, reinterpret_cast<uint32_t*>(p.out), p.ldo, grow - lane, p.rows,
                                  tn * p.bn + rank * slice + ci * 16, p.cols, p.vec_out, s_stage);
              continue;
            }
            uint32_t own[16], v[16];
            __syncwarp();
            tmem_ld16(tbase + rank * slice + ci * 16, own);
            tmem_ld_wait();
            #pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = 0u;
            for (int q = 0; q < S; ++q) {
              const uint32_t* src = recv + ((q - (q > rank ? 1 : 0)) * slice + ci * 16) * kTileRows + row;
              #pragma unroll
              for (int j = 0; j < 16; ++j) {
                const uint32_t a = (q == rank) ? own[j] : src[j * kTileRows];
                if constexpr (kInt)
                  v[j] += a;
                else
                  v[j] = __float_as_uint(__fadd_rn(__uint_as_float(v[j]), __uint_as_float(a)));
              }
            }
            const int c = rank * slice + ci * 16;
            epi_norm16<MODE>(p, grow - lane, tn * p.bn + c, v, s_stage, reinterpret_cast<const float*>(s_exp) + c);
          }
          release_accum();
          epi_cluster_done = true;
          if (trace) {
            epi_fin += globaltimer() - tp2;
            epi_items += 1;
          }
          continue;
        }
      }

      // Split tile of a swap mode (stream-K). The slot is column-major
      // ([tok][128 rows], a warp's 32 rows of one token contiguous). Every
      // contributor adds one combined value per real token atomically into the
      // slot of the CTA that holds the tile's last unit; the CTA whose count
      // completes the tile reads the slot, clears it and finishes the tile.
      if constexpr (kSwap) {
        const long long tile_u0 = static_cast<long long>(w.tile) * sc.kb_tile;
        const int slot = sc.owner(tile_u0 + sc.kb_tile - 1);
        using SV = typename SwapVal<MODE>::T;
        SV* vcol = reinterpret_cast<SV*>(p.slots + static_cast<long long>(slot) * kTileRows * p.bn) + row;
        for (int ci = half; ci < nch; ci += 2) {
          const int c = ci * kChunk;
          uint32_t v[48];
          __syncwarp();
          tmem_ld16(tbase + c, *reinterpret_cast<uint32_t(*)[16]>(v));
          tmem_ld16(tbase + c + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
          tmem_ld16(tbase + c + 32, *reinterpret_cast<uint32_t(*)[16]>(v + 32));
          tmem_ld_wait();
          #pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int lt = c / 3 + j;
            if (tok0 + lt < p.n_tokens) atomicAdd(vcol + lt * kTileRows, swap_combine<MODE>(v + 3 * j));
          }
        }
        release_accum();
        // The barrier orders every epilogue thread's slot writes before thread
        // 0's release-acquire count; the finisher's acquire plus the second
        // barrier make all contributors' writes visible to its threads.
        named_bar_sync(1, kEpiThreads);
        const unsigned long long tp1 = trace ? globaltimer() : 0;
        if (trace) epi_pub += tp1 - tp0;
        if (ethread == 0) {
          const int done = atom_add_acq_rel_gpu(p.counters + w.tile, w.kb1 - w.kb0) + (w.kb1 - w.kb0);
          const int last = (done == sc.kb_tile);
          if (last) p.counters[w.tile] = 0;  // ready for the next call
          *bcast = last;
        }
        named_bar_sync(1, kEpiThreads);
        const unsigned long long tp2 = trace ? globaltimer() : 0;
        if (trace) epi_cnt += tp2 - tp1;
        const int last = *bcast;
        if (!last) continue;
        const int ntok = min(p.tok_per_tile, p.n_tokens - tok0);
        for (int lt0 = half * 8; lt0 < ntok; lt0 += 16) {
          SV vals[8];
          #pragma unroll
          for (int j = 0; j < 8; ++j) vals[j] = (lt0 + j < ntok) ? __ldcg(vcol + (lt0 + j) * kTileRows) : SV(0);
          #pragma unroll
          for (int j = 0; j < 8; ++j)
            if (lt0 + j < ntok) __stcg(vcol + (lt0 + j) * kTileRows, SV(0));
          if (grow < p.n_out) {
            #pragma unroll
            for (int j = 0; j < 8; ++j)
              if (lt0 + j < ntok)
                swap_finish<MODE>(p, grow, tok0 + lt0 + j, lt0 + j, vals[j], scale_n, s_exp, s_bad);
          }
        }
        if (trace) {
          epi_fin += globaltimer() - tp2;
          epi_items += 1;
        }
      }
    }
  }

  // A cluster-split launch: every thread takes the two cluster barrier steps
  // exactly once (warps 0 and 1 here; epilogue threads that gave up waiting
  // for their accumulator too), so no CTA waits for a thread that left.
  if (p.csplit > 1) {
    bool todo = warp < 2;
    if (warp >= 2) todo = !epi_cluster_done;
    if (warp < 2) __syncwarp();
    if (todo) {
      cluster_arrive_release();
      cluster_wait_acquire();
      cluster_arrive_release();
      cluster_wait_acquire();
    }
  }

  // Teardown: every role has left its loop (normally or on abort). The
  // epilogue warps report on done_bar; the TMEM owner waits for all four
  // before releasing TMEM (a CTA-wide barrier is not used here because warps
  // 0 and 1 reach it from divergent single-lane loops).
  if (warp >= 2) {
    if (trace && threadIdx.x == 64) {
      trace[6] = globaltimer();
      trace[11] = epi_wait;
      trace[12] = epi_pub;
      trace[13] = epi_cnt;
      trace[14] = epi_fin;
      trace[15] = epi_items;
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(done_bar);
  }
  if (warp == 1) {
    __syncwarp();
    mbar_wait(done_bar, 0, p.err, abort_flag, kDevTimeoutDrain, false);
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem_base, p.tmem_cols);
    if (trace && lane == 0) trace[7] = globaltimer();
  }

  // Row-sharded call: after this rank's last CTA has stored its outputs into
  // every rank's C, every rank's inbox gets 1; the kernel ends when this rank's
  // inbox holds all ranks' counts for this call (bounded wait). This follows
  // the TMEM release, so the wait holds no tensor-core resources.
  if (p.npeers > 0 && warp >= 2) {
    fence_sc_sys();  // this thread's peer stores are visible before the counts below
    named_bar_sync(1, kEpiThreads);
    if (threadIdx.x == 64) {
      const unsigned done = static_cast<unsigned>(atom_add_acq_rel_gpu(p.done_ctr, 1u)) + 1u;
      if (done == gridDim.x) {
        *p.done_ctr = 0u;  // ready for the next call
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

// Row-sharded calls gathered by copy engines: a peer's count, added once this
// rank's copies into the peer's C are done (the kernel follows them on the
// copy stream), and the bounded wait for every rank's count of a call.
__global__ void peer_signal_kernel(unsigned* inbox) {
  if (threadIdx.x == 0) {
    fence_sc_sys();
    red_add_release_sys(inbox, 1u);
  }
}

// Row-sharded calls on more than two GPUs: push rows [0, rows) x columns
// [0, cols) of this rank's slice of C (src, row pitch ld floats) into the same
// place of every other rank's C (dst.p[q], q != self) with plain stores over
// NVLink, a grid-stride loop over 16-byte vectors (vec) or single floats. It
// runs beside the GEMM's next row chunk (a few registers, no shared memory, so
// its CTAs fit next to the GEMM's). Then every rank's inbox gets one count from
// peer_signal_all_kernel.
struct PeerDst {
  float* p[kMaxPeers];
  unsigned* inbox[kMaxPeers];
};

__global__ void __launch_bounds__(256) peer_push_kernel(const float* __restrict__ src, long long ld, int rows, int cols,
                                                        const __grid_constant__ PeerDst dst, int npeers, int self,
                                                        int vec) {
  const long long nth = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    const int c4 = cols / 4;
    const long long total = static_cast<long long>(rows) * c4;
    for (long long i = tid; i < total; i += nth) {
      const long long r = i / c4;
      const long long off = r * ld + (i - r * c4) * 4;
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + off));
      for (int q = 0; q < npeers; ++q)
        if (q != self) *reinterpret_cast<float4*>(dst.p[q] + off) = v;
    }
  } else {
    const long long total = static_cast<long long>(rows) * cols;
    for (long long i = tid; i < total; i += nth) {
      const long long r = i / cols;
      const long long off = r * ld + (i - r * cols);
      const float v = __ldcg(src + off);
      for (int q = 0; q < npeers; ++q)
        if (q != self) dst.p[q][off] = v;
    }
  }
}

// One count in every other rank's inbox, after all of this rank's stores into
// their C (the kernels before it in the stream) are visible to them.
__global__ void peer_signal_all_kernel(const __grid_constant__ PeerDst dst, int npeers, int self) {
  const int q = static_cast<int>(threadIdx.x);
  if (q < npeers && q != self) {
    fence_sc_sys();
    red_add_release_sys(dst.inbox[q], 1u);
  }
}

__global__ void peer_wait_kernel(const unsigned* inbox, unsigned target, int* err) {
  if (threadIdx.x != 0) return;
  const unsigned long long t0 = globaltimer();
  while (static_cast<int>(ld_acquire_sys(inbox) - target) < 0) {
    if (globaltimer() - t0 > kPeerWaitLimitNs) {
      atomicCAS(err, 0, kDevTimeoutPeers);
      return;
    }
    __nanosleep(256);
  }
}

}  // namespace vmlm
