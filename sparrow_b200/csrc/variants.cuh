// variants.cuh -- the weight-quantisation variants of the reference's study
// (tests/src/quant.rs): int4 weights with an f32 scale per group of columns
// (:114-152, :298-362), and the int8 GEMM whose outlier input columns are
// added back in f32 (LLM.int8, :458-565). Decode-size GEMMs: CUDA-core kernels
// that stream the packed weights once.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "prep.cuh"
#include "ptx.cuh"

namespace vmlm {

constexpr int kDevIdxRange = 103;  // an outlier column index >= k

// ------------------------------------------------------------ int4 grouped
//
// Layout (tests/src/quant.rs:114-152): rows of (k+1)/2 bytes, column p in the
// low nibble of byte p/2 when p is even and the high nibble when odd, two's
// complement in [-8, 7]; scale [n][gpr], gpr = ceil(k/group).
//
// The reference's AVX2 step (:316-333) does not read that order: a 32-column
// step at column kk loads 16 bytes at kk/2 into both 128-bit halves, so its
// unpacks repeat bytes 0-3 and 8-11, and it takes each byte's high nibble
// first. Column kk+t (t < 32) uses the nibble of byte kk/2 + (t&16)/2 +
// (t&7)/2, high when t is even. Only 32-column steps that fit inside a group
// do that; the rest of a group (its scalar tail) follows the packed order.
// `order` 1 reproduces the step as shipped, 0 uses the packed order.

constexpr int kI4Warps = 8;
constexpr int kI4SmemFloats = 24576;  // 96 KB of staged activations per CTA
constexpr int kI4LanesPerRow = 8;     // a weight row's 32-column units go to 8 lanes
constexpr int kI4RowsPerBlock = kI4Warps * 32 / kI4LanesPerRow;

// Swap the two nibbles of every byte.
__device__ __forceinline__ uint32_t nib_swap(uint32_t w) { return ((w >> 4) & 0x0F0F0F0Fu) | ((w & 0x0F0F0F0Fu) << 4); }

// Column class c = p % 8 of a 32-column unit: its nibble sits at bits sh = 4c
// of the word for c < 5 and at bits sh = 4c - 12 of the word shifted right by
// 12 for c >= 5 (sh <= 16). One LOP3 per column, (src & (0xF << sh)) ^
// (0x4B000000 | 8 << sh), gives the float f = 2^23 + (nibble ^ 8) * 2^sh, and
// f - (2^23 + 8 * 2^sh) = v * 2^sh exactly (v the signed nibble). The staged
// activations carry the factor 2^-sh, so a' * (v 2^sh) = a * v with the same
// rounding (power-of-two scaling is exact).
__host__ __device__ constexpr int i4_shift(int c) { return c < 5 ? 4 * c : 4 * c - 12; }

__device__ __forceinline__ float i4_val(uint32_t w, uint32_t w12, int c) {
  const uint32_t src = c < 5 ? w : w12;
  const int sh = i4_shift(c);
  const float f = __uint_as_float((src & (0xFu << sh)) ^ (0x4B000000u | (0x8u << sh)));
  return f - (8388608.0f + 8.0f * static_cast<float>(1 << sh));
}

// Fast path: k % 32 == 0, group % 32 == 0, 16-byte aligned rows (so every
// 32-column unit lies inside one group and is one reference step). Grid
// (row-set CTAs, ceil(m / MB)); lane l of a warp works on weight row
// 4 * warp + l / 8 of the CTA's row set and takes its units l % 8, l % 8 + 8,
// ..., the next unit's weights loaded before the current one is computed. The
// activations of MB token rows are staged in shared memory in chunks of kc
// columns, a unit's eight float4 at a stride of nine float4 per unit: the
// eight units a warp reads at once hit eight different bank groups, the four
// lanes on the same unit (one per weight row) read the same words
// (broadcast), and a unit's reads are one base address plus constants.
template <int MB, int ORDER>
__global__ void __launch_bounds__(kI4Warps * 32) int4gs_kernel(const float* __restrict__ a,
                                                               const uint8_t* __restrict__ packed,
                                                               const float* __restrict__ scale, float* __restrict__ c,
                                                               int m, int n, int k, int group, int gpr, int kc) {
  extern __shared__ float4 s_a4[];
  pdl_launch_dependents();
  pdl_wait_prior();
  const int m0 = blockIdx.y * MB;
  const int rows_m = m - m0 < MB ? m - m0 : MB;
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int u0 = lane % kI4LanesPerRow;
  const long long rowbytes = k / 2;
  const int rs = kc / 32 * 9;  // float4 per staged token row
  const bool one_chunk = kc >= k;

  auto stage = [&](int kc0, int kcn) {
    // a'[r][p] = a[m0 + r][kc0 + p] * 2^-(i4_shift(p % 8)); rows past m are zero.
    // float4 f covers columns 4f .. 4f+3 (classes 0-3 or 4-7 of its unit).
    const int kcn4 = kcn / 4;
    constexpr int kUnroll = 4;
    for (int e0 = static_cast<int>(threadIdx.x); e0 < MB * kcn4; e0 += kUnroll * blockDim.x) {
      float4 v[kUnroll];
#pragma unroll
      for (int q = 0; q < kUnroll; ++q) {
        const int e = e0 + q * static_cast<int>(blockDim.x);
        const int r = e / kcn4, f = e - r * kcn4;
        v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e < MB * kcn4 && r < rows_m)
          v[q] = __ldg(reinterpret_cast<const float4*>(a + static_cast<long long>(m0 + r) * k + kc0) + f);
      }
#pragma unroll
      for (int q = 0; q < kUnroll; ++q) {
        const int e = e0 + q * static_cast<int>(blockDim.x);
        if (e >= MB * kcn4) break;
        const int r = e / kcn4, f = e - r * kcn4;
        const int c0 = (f & 1) * 4;  // column class of the float4's first column
        float4 x = v[q];
        x.x *= __uint_as_float(static_cast<uint32_t>(127 - i4_shift(c0)) << 23);
        x.y *= __uint_as_float(static_cast<uint32_t>(127 - i4_shift(c0 + 1)) << 23);
        x.z *= __uint_as_float(static_cast<uint32_t>(127 - i4_shift(c0 + 2)) << 23);
        x.w *= __uint_as_float(static_cast<uint32_t>(127 - i4_shift(c0 + 3)) << 23);
        s_a4[r * rs + (f >> 3) * 9 + (f & 7)] = x;
      }
    }
  };

  if (one_chunk) {
    stage(0, k);
    __syncthreads();
  }
  for (int j0 = blockIdx.x * kI4RowsPerBlock; j0 < n; j0 += gridDim.x * kI4RowsPerBlock) {
    const int jwarp = j0 + warp * (32 / kI4LanesPerRow);
    const int j = jwarp + lane / kI4LanesPerRow;
    const int jr = j < n ? j : n - 1;  // a past-the-end row reads row n-1 and is not stored
    float tot[MB];
#pragma unroll
    for (int i = 0; i < MB; ++i) tot[i] = 0.f;
    for (int kc0 = 0; kc0 < k; kc0 += kc) {
      const int kcn = k - kc0 < kc ? k - kc0 : kc;
      if (!one_chunk) {
        __syncthreads();
        stage(kc0, kcn);
        __syncthreads();
      }
      const int units = kcn / 32;
      if (jwarp < n && u0 < units) {
        const uint4* wrow = reinterpret_cast<const uint4*>(packed + jr * rowbytes) + kc0 / 32;
        const float* srow = scale + static_cast<long long>(jr) * gpr;
        uint4 wv = __ldg(wrow + u0);
        float sc = __ldg(srow + (kc0 + u0 * 32) / group);
        for (int u = u0; u < units; u += kI4LanesPerRow) {
          uint4 wn = wv;
          float sn = sc;
          if (u + kI4LanesPerRow < units) {
            wn = __ldg(wrow + u + kI4LanesPerRow);
            sn = __ldg(srow + (kc0 + (u + kI4LanesPerRow) * 32) / group);
          }
          if (ORDER == 1) {
            const uint32_t x0 = nib_swap(wv.x), x2 = nib_swap(wv.z);
            wv = make_uint4(x0, x0, x2, x2);
          }
          const float4* sa = s_a4 + u * 9;
          float part[MB];
#pragma unroll
          for (int i = 0; i < MB; ++i) part[i] = 0.f;
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const uint32_t w = (v >> 1) == 0 ? wv.x : (v >> 1) == 1 ? wv.y : (v >> 1) == 2 ? wv.z : wv.w;
            const uint32_t w12 = w >> 12;
            const int c0 = (v & 1) * 4;
            const float d0 = i4_val(w, w12, c0), d1 = i4_val(w, w12, c0 + 1);
            const float d2 = i4_val(w, w12, c0 + 2), d3 = i4_val(w, w12, c0 + 3);
#pragma unroll
            for (int i = 0; i < MB; ++i) {
              const float4 av = sa[i * rs + v];
              float s = part[i];
              s = fmaf(av.x, d0, s);
              s = fmaf(av.y, d1, s);
              s = fmaf(av.z, d2, s);
              s = fmaf(av.w, d3, s);
              part[i] = s;
            }
          }
#pragma unroll
          for (int i = 0; i < MB; ++i) tot[i] = fmaf(part[i], sc, tot[i]);
          wv = wn;
          sc = sn;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < MB; ++i) {
      float s = tot[i];
#pragma unroll
      for (int o = kI4LanesPerRow / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (u0 == 0 && j < n && i < rows_m) c[static_cast<long long>(m0 + i) * n + j] = s;
    }
  }
}

// Integer form for one or two token rows (the HBM-bound case), same tile rules
// and lane mapping as int4gs_kernel, one token row per grid row (blockIdx.y).
// The token row becomes three int8 digit planes of its 22-bit fixed-point
// form X = rint(x * 2^e) (one exponent per row, as the Q8 path makes them), and
// each weight nibble the unsigned byte u = nibble ^ 8 = v + 8: per 8 columns
// one LOP3 and one shift + LOP3 give the bytes of the even and of the odd
// columns, and two dp4a per plane add u * X_p. A 32-column unit's sum is then
// sum_p 256^p (D_p - 8 sum X_p), exactly sum X * v (|.| <= 2^30), converted
// once to f32 and multiplied by the group's scale; the row total is scaled by
// 2^-e at the end. Staged per unit (7 uint4, 112 bytes, stride 7 so eight
// consecutive units fall in eight bank groups): even-column and odd-column
// plane words of planes 0, 1, 2, then the unit's digit sums. A row holding NaN
// or Inf is computed in f32 instead (the row staged as floats, scalar decode).
constexpr int kI4UnitWords = 7;

template <int ORDER>
__global__ void __launch_bounds__(kI4Warps * 32) int4gs_dp4a_kernel(const float* __restrict__ a,
                                                                    const uint8_t* __restrict__ packed,
                                                                    const float* __restrict__ scale,
                                                                    float* __restrict__ c, int n, int k, int group,
                                                                    int gpr, int kc) {
  extern __shared__ uint4 s_u[];
  __shared__ float redf[32];
  __shared__ int redi[32];
  pdl_launch_dependents();
  pdl_wait_prior();
  const int t = blockIdx.y;
  const float* xr = a + static_cast<long long>(t) * k;
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int u0 = lane % kI4LanesPerRow;
  const long long rowbytes = k / 2;
  const int ukc = kc / 32;                          // units per staged chunk
  float* s_x = reinterpret_cast<float*>(s_u + ukc * kI4UnitWords);  // f32 row chunk (NaN/Inf rows only)
  const bool one_chunk = kc >= k;

  // the row's exponent and non-finite flag over the whole K
  float amax = 0.f;
  int bad = 0;
  for (int i = static_cast<int>(threadIdx.x); i < k / 4; i += blockDim.x) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(xr) + i);
    bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  block_max_or(amax, bad, redf, redi);
  int e = 0;
  if (!bad && amax > 0.f) {
    int E;
    frexpf(amax, &E);
    e = 22 - E;
  }

  auto stage = [&](int kc0, int kcn) {
    if (bad) {
      for (int i = static_cast<int>(threadIdx.x); i < kcn / 4; i += blockDim.x)
        reinterpret_cast<float4*>(s_x)[i] = __ldg(reinterpret_cast<const float4*>(xr + kc0) + i);
      return;
    }
    // thread per 8-column word q (units of 4 words); the 4 threads of a unit are
    // consecutive lanes and combine their digit sums by shuffles
    const int nw = kcn / 8;
    for (int q0 = 0; q0 < nw; q0 += blockDim.x) {
      const int q = q0 + static_cast<int>(threadIdx.x);
      int sx[3] = {0, 0, 0};
      if (q < nw) {
        const float4 v0 = __ldg(reinterpret_cast<const float4*>(xr + kc0) + 2 * q);
        const float4 v1 = __ldg(reinterpret_cast<const float4*>(xr + kc0) + 2 * q + 1);
        const float xs[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        int d[3][8];
        #pragma unroll
        for (int j = 0; j < 8; ++j) {
          q8_digits(xs[j], e, d[0][j], d[1][j], d[2][j]);
          sx[0] += d[0][j];
          sx[1] += d[1][j];
          sx[2] += d[2][j];
        }
        uint32_t* su = reinterpret_cast<uint32_t*>(s_u + (q >> 2) * kI4UnitWords);
        #pragma unroll
        for (int p = 0; p < 3; ++p) {
          su[(2 * p) * 4 + (q & 3)] = pack4(d[p][0], d[p][2], d[p][4], d[p][6]);
          su[(2 * p + 1) * 4 + (q & 3)] = pack4(d[p][1], d[p][3], d[p][5], d[p][7]);
        }
      }
      #pragma unroll
      for (int p = 0; p < 3; ++p) {
        sx[p] += __shfl_xor_sync(0xffffffffu, sx[p], 1);
        sx[p] += __shfl_xor_sync(0xffffffffu, sx[p], 2);
      }
      if (q < nw && (q & 3) == 0) s_u[(q >> 2) * kI4UnitWords + 6] = make_uint4(sx[0], sx[1], sx[2], 0);
    }
  };

  // one 32-column unit of weight row j: sum X * v as a float (or the f32 sum of
  // a NaN/Inf row), before the group's scale
  auto unit_value = [&](uint4 wv, int u) -> float {
    if (ORDER == 1) {
      const uint32_t x0 = nib_swap(wv.x), x2 = nib_swap(wv.z);
      wv = make_uint4(x0, x0, x2, x2);
    }
    const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
    if (!bad) {
      const uint4* su = s_u + u * kI4UnitWords;
      const uint4 e0 = su[0], o0 = su[1], e1 = su[2], o1 = su[3], e2 = su[4], o2 = su[5], sx = su[6];
      const uint32_t E0[4] = {e0.x, e0.y, e0.z, e0.w}, O0[4] = {o0.x, o0.y, o0.z, o0.w};
      const uint32_t E1[4] = {e1.x, e1.y, e1.z, e1.w}, O1[4] = {o1.x, o1.y, o1.z, o1.w};
      const uint32_t E2[4] = {e2.x, e2.y, e2.z, e2.w}, O2[4] = {o2.x, o2.y, o2.z, o2.w};
      int D0 = 0, D1 = 0, D2 = 0;
      #pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int lo = static_cast<int>((ws[i] & 0x0F0F0F0Fu) ^ 0x08080808u);
        const int hi = static_cast<int>(((ws[i] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u);
        D0 = __dp4a(lo, static_cast<int>(E0[i]), D0);
        D0 = __dp4a(hi, static_cast<int>(O0[i]), D0);
        D1 = __dp4a(lo, static_cast<int>(E1[i]), D1);
        D1 = __dp4a(hi, static_cast<int>(O1[i]), D1);
        D2 = __dp4a(lo, static_cast<int>(E2[i]), D2);
        D2 = __dp4a(hi, static_cast<int>(O2[i]), D2);
      }
      const int S = (D0 - 8 * static_cast<int>(sx.x)) + 256 * (D1 - 8 * static_cast<int>(sx.y)) +
                    65536 * (D2 - 8 * static_cast<int>(sx.z));
      return __int2float_rn(S);
    }
    const float* xs = s_x + u * 32;
    float part = 0.f;
    #pragma unroll
    for (int cidx = 0; cidx < 32; ++cidx) {
      const uint32_t nib = (ws[cidx >> 3] >> (4 * (cidx & 7))) & 15u;
      part = fmaf(xs[cidx], static_cast<float>(static_cast<int>(nib) - (nib > 7 ? 16 : 0)), part);
    }
    return part;
  };
  auto finish_row = [&](float tot, int j) {
    #pragma unroll
    for (int o = kI4LanesPerRow / 2; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if (u0 == 0 && j < n) c[static_cast<long long>(t) * n + j] = bad ? tot : scale_pow2(tot, -e);
  };
  const int rows_step = gridDim.x * kI4RowsPerBlock;

  if (one_chunk) {
    stage(0, k);
    __syncthreads();
    // one flat stream per lane over (row set, step): the weight loads run two
    // steps ahead across row-set boundaries, so a row set's first loads do not
    // start cold; a row's total is reduced and stored after its last step
    const int units = k / 32;
    const int steps = (units + kI4LanesPerRow - 1) / kI4LanesPerRow;
    const int jlane = warp * (32 / kI4LanesPerRow) + lane / kI4LanesPerRow;  // row within a row set
    auto fetch = [&](int j0, int st, uint4& w, float& s) {
      const int u = u0 + st * kI4LanesPerRow;
      const int j = j0 + jlane;
      if (j0 < n && u < units) {
        const int jr = j < n ? j : n - 1;
        w = __ldg(reinterpret_cast<const uint4*>(packed + jr * rowbytes) + u);
        s = __ldg(scale + static_cast<long long>(jr) * gpr + u * 32 / group);
      }
    };
    int j0 = blockIdx.x * kI4RowsPerBlock, st = 0;   // current position
    int pj = j0, pst = 0;                              // next position to fetch
    uint4 w0 = make_uint4(0, 0, 0, 0), w1 = w0;
    float s0 = 0.f, s1 = 0.f;
    auto advance = [&](int& jj, int& ss) {
      if (++ss == steps) {
        ss = 0;
        jj += rows_step;
      }
    };
    fetch(pj, pst, w0, s0);
    advance(pj, pst);
    fetch(pj, pst, w1, s1);
    advance(pj, pst);
    float tot = 0.f;
    while (j0 < n) {
      uint4 w2 = w1;
      float s2 = s1;
      fetch(pj, pst, w2, s2);
      advance(pj, pst);
      const int u = u0 + st * kI4LanesPerRow;
      if (u < units) tot = fmaf(unit_value(w0, u), s0, tot);  // rows past n hold row n-1 and are not stored
      if (st == steps - 1) {
        finish_row(tot, j0 + jlane);
        tot = 0.f;
      }
      advance(j0, st);
      w0 = w1;
      s0 = s1;
      w1 = w2;
      s1 = s2;
    }
    return;
  }
  for (int j0 = blockIdx.x * kI4RowsPerBlock; j0 < n; j0 += rows_step) {
    const int jwarp = j0 + warp * (32 / kI4LanesPerRow);
    const int j = jwarp + lane / kI4LanesPerRow;
    const int jr = j < n ? j : n - 1;  // a past-the-end row reads row n-1 and is not stored
    float tot = 0.f;
    for (int kc0 = 0; kc0 < k; kc0 += kc) {
      const int kcn = k - kc0 < kc ? k - kc0 : kc;
      __syncthreads();
      stage(kc0, kcn);
      __syncthreads();
      const int units = kcn / 32;
      if (jwarp < n && u0 < units) {
        const uint4* wrow = reinterpret_cast<const uint4*>(packed + jr * rowbytes) + kc0 / 32;
        const float* srow = scale + static_cast<long long>(jr) * gpr;
        for (int u = u0; u < units; u += kI4LanesPerRow)
          tot = fmaf(unit_value(__ldg(wrow + u), u), __ldg(srow + (kc0 + u * 32) / group), tot);
      }
    }
    finish_row(tot, j);
  }
}

// Any shape: a warp per (token row, weight row), lanes over columns. The lane
// sums its columns of one group, then adds that sum times the group's scale.
template <int ORDER>
__global__ void __launch_bounds__(256) int4gs_generic_kernel(const float* __restrict__ a,
                                                             const uint8_t* __restrict__ packed,
                                                             const float* __restrict__ scale, float* __restrict__ c,
                                                             int m, int n, int k, int group, int gpr) {
  pdl_launch_dependents();
  pdl_wait_prior();
  const long long wid = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  if (wid >= static_cast<long long>(m) * n) return;
  const int i = static_cast<int>(wid / n), j = static_cast<int>(wid - static_cast<long long>(i) * n);
  const uint8_t* pr = packed + static_cast<long long>(j) * ((k + 1) / 2);
  const float* ar = a + static_cast<long long>(i) * k;
  float tot = 0.f, part = 0.f;
  int gcur = -1;
  for (int p = lane; p < k; p += 32) {
    const int g = p / group;
    if (g != gcur) {
      if (gcur >= 0) tot = fmaf(part, __ldg(scale + static_cast<long long>(j) * gpr + gcur), tot);
      part = 0.f;
      gcur = g;
    }
    int byte, hi;
    const int gs = g * group;
    const int gend = gs + group < k ? gs + group : k;
    const int bs = gs + (p - gs) / 32 * 32;
    if (ORDER == 1 && bs + 32 <= gend) {
      const int t = p - bs;
      byte = bs / 2 + ((t & 16) >> 1) + ((t & 7) >> 1);
      hi = (t & 1) == 0;
    } else {
      byte = p / 2;
      hi = p & 1;
    }
    const uint32_t bv = __ldg(pr + byte);
    const int nib = hi ? (bv >> 4) & 15 : bv & 15;
    part = fmaf(__ldg(ar + p), static_cast<float>(nib > 7 ? nib - 16 : nib), part);
  }
  if (gcur >= 0) tot = fmaf(part, __ldg(scale + static_cast<long long>(j) * gpr + gcur), tot);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  if (lane == 0) c[static_cast<long long>(i) * n + j] = tot;
}

// ------------------------------------------------- int8 + outlier columns
//
// After the int8 GEMM has written c (tests/src/quant.rs:524-565 computes the
// int8 body times scale first), c[i][j] += a[i][idx[t]] * w(j, t) for t in list
// order, each product rounded and then added, as the reference does. w(j, t)
// is wo[j * n_idx + t] for the compact outlier matrix, or w[j * k + idx[t]]
// for the full f32 weight. A thread per weight row j and kOutRows token rows;
// the listed activation columns are staged in shared memory kOutChunk at a
// time. An index >= k records kDevIdxRange and adds nothing for that entry.
constexpr int kOutRows = 8;
constexpr int kOutChunk = 512;

__global__ void __launch_bounds__(256) outlier_add_kernel(const float* __restrict__ a, const float* __restrict__ w,
                                                          int compact, const uint32_t* __restrict__ idx, int n_idx,
                                                          float* __restrict__ c, int m, int n, int k,
                                                          int* __restrict__ err) {
  __shared__ float s_a[kOutRows][kOutChunk];
  __shared__ int s_ok[kOutChunk];
  pdl_launch_dependents();
  pdl_wait_prior();
  const int m0 = blockIdx.y * kOutRows;
  const int rows_m = m - m0 < kOutRows ? m - m0 : kOutRows;
  const int j = blockIdx.x * blockDim.x + static_cast<int>(threadIdx.x);
  float v[kOutRows];
#pragma unroll
  for (int r = 0; r < kOutRows; ++r) v[r] = (j < n && r < rows_m) ? c[static_cast<long long>(m0 + r) * n + j] : 0.f;
  for (int t0 = 0; t0 < n_idx; t0 += kOutChunk) {
    const int tn = n_idx - t0 < kOutChunk ? n_idx - t0 : kOutChunk;
    __syncthreads();
    for (int e = static_cast<int>(threadIdx.x); e < tn; e += blockDim.x) {
      const uint32_t col = __ldg(idx + t0 + e);
      const int ok = col < static_cast<uint32_t>(k);
      s_ok[e] = ok;
      if (!ok && blockIdx.x == 0 && blockIdx.y == 0) atomicCAS(err, 0, kDevIdxRange);
      for (int r = 0; r < kOutRows; ++r)
        s_a[r][e] = (ok && r < rows_m) ? __ldg(a + static_cast<long long>(m0 + r) * k + col) : 0.f;
    }
    __syncthreads();
    if (j < n) {
      for (int t = 0; t < tn; ++t) {
        if (!s_ok[t]) continue;
        const float wj = compact ? __ldg(w + static_cast<long long>(j) * n_idx + t0 + t)
                                 : __ldg(w + static_cast<long long>(j) * k + __ldg(idx + t0 + t));
#pragma unroll
        for (int r = 0; r < kOutRows; ++r) v[r] = __fadd_rn(v[r], __fmul_rn(s_a[r][t], wj));
      }
    }
  }
  if (j < n)
#pragma unroll
    for (int r = 0; r < kOutRows; ++r)
      if (r < rows_m) c[static_cast<long long>(m0 + r) * n + j] = v[r];
}

// wo[j][t] = w[j][idx[t]]: the compact outlier matrix [n][n_idx], built once per
// weight. An index >= k records kDevIdxRange and writes 0.
__global__ void __launch_bounds__(256) gather_columns_kernel(const float* __restrict__ w,
                                                             const uint32_t* __restrict__ idx, int n_idx,
                                                             float* __restrict__ wo, int n, int k,
                                                             int* __restrict__ err) {
  const long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= static_cast<long long>(n) * n_idx) return;
  const int j = static_cast<int>(e / n_idx), t = static_cast<int>(e - static_cast<long long>(j) * n_idx);
  const uint32_t col = __ldg(idx + t);
  if (col >= static_cast<uint32_t>(k)) {
    atomicCAS(err, 0, kDevIdxRange);
    wo[e] = 0.f;
    return;
  }
  wo[e] = __ldg(w + static_cast<long long>(j) * k + col);
}

}  // namespace vmlm
