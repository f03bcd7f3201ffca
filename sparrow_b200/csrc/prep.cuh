// prep.cuh -- activation preparation kernels and CUDA-core kernels for shapes
// the TMA path cannot take (K not a multiple of 16 bytes, unaligned rows).
//
// Q8 activations are encoded as three signed 8-bit digit planes per token:
//   e   = 22 - E  where max|x_t| = f * 2^E, f in [0.5, 1)   (e = 0 for a zero row)
//   X   = rint(x * 2^e)              |X| <= 2^22; the power-of-two scaling is exact
//   X   = d0 + 256*d1 + 65536*d2     d0, d1 in [-128,127], d2 in [-64,64]
// so sum_k x_k*q_k = 2^-e * sum_p 256^p * (sum_k d_p,k * q_k) up to the
// 2^-23*max|x| rounding of X; the three int32 sums are exact.
//
// bf16 activations (f32 in, bf16 weights) are split into three bf16 terms
//   hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)
// (each difference is exact in f32), which carry 24 significant bits.
//
// Both kernels run one CTA per token and keep the row in registers (up to
// kPrepThreads * kPrepVec elements; longer rows are read twice), with one
// block reduction for the row's flags.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace vmlm {

constexpr int kPrepThreads = 512;
constexpr int kPrepVec = 16;  // elements per thread kept in registers (4 float4)

__device__ __forceinline__ float warp_max(float v) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_or(int v) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide max of a float and OR of an int in one pass (two shared arrays).
__device__ __forceinline__ void block_max_or(float& m, int& o, float* redf, int* redi) {
  m = warp_max(m);
  o = warp_or(o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    redf[w] = m;
    redi[w] = o;
  }
  __syncthreads();
  const int nw = blockDim.x >> 5;
  m = (l < nw) ? redf[l] : 0.f;
  o = (l < nw) ? redi[l] : 0;
  m = warp_max(m);
  o = warp_or(o);
}

__device__ __forceinline__ int block_or(int v, int* red) {
  v = warp_or(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = (l < static_cast<int>(blockDim.x >> 5)) ? red[l] : 0;
  return warp_or(v);
}

// x * 2^e for exponents outside the normal range of a single 2^e factor (out
// of line, so the callers' unrolled loops stay small).
__device__ __noinline__ float scale_pow2_wide(float x, int e) { return scalbnf(x, e); }

// x * 2^e exactly (power-of-two scaling), for any e the encoder produces.
__device__ __forceinline__ float scale_pow2(float x, int e) {
  if (e >= -126 && e <= 127) return __fmul_rn(x, __int_as_float((127 + e) << 23));
  return scale_pow2_wide(x, e);
}

__device__ __forceinline__ void q8_digits(float x, int e, int& d0, int& d1, int& d2) {
  const int X = __float2int_rn(scale_pow2(x, e));
  d0 = ((X + 128) & 255) - 128;
  const int X1 = (X - d0) >> 8;
  d1 = ((X1 + 128) & 255) - 128;
  d2 = (X1 - d1) >> 8;
}

// The three digit planes of four values at once, packed (byte j of plane p =
// digit p of element j, as pack4 of q8_digits). With X = rint(x * 2^e),
// |X| <= 2^22, Y = X + 0x808080 is positive and its bytes 0, 1, 2 are the
// balanced digits d0, d1, d2 plus 128 each (the carries of the balanced form
// are those of adding 128 to each byte), so each plane byte is a byte of Y
// with its top bit flipped: three byte permutes per plane pair instead of
// the digit arithmetic per element.
__device__ __forceinline__ void q8_digits4(float4 v, int e, uint32_t& p0, uint32_t& p1, uint32_t& p2) {
  const uint32_t ya = static_cast<uint32_t>(__float2int_rn(scale_pow2(v.x, e)) + 0x808080);
  const uint32_t yb = static_cast<uint32_t>(__float2int_rn(scale_pow2(v.y, e)) + 0x808080);
  const uint32_t yc = static_cast<uint32_t>(__float2int_rn(scale_pow2(v.z, e)) + 0x808080);
  const uint32_t yd = static_cast<uint32_t>(__float2int_rn(scale_pow2(v.w, e)) + 0x808080);
  const uint32_t ab01 = __byte_perm(ya, yb, 0x5140);  // a0 b0 a1 b1
  const uint32_t cd01 = __byte_perm(yc, yd, 0x5140);  // c0 d0 c1 d1
  const uint32_t ab2 = __byte_perm(ya, yb, 0x0062);   // a2 b2 . .
  const uint32_t cd2 = __byte_perm(yc, yd, 0x0062);   // c2 d2 . .
  p0 = __byte_perm(ab01, cd01, 0x5410) ^ 0x80808080u;
  p1 = __byte_perm(ab01, cd01, 0x7632) ^ 0x80808080u;
  p2 = __byte_perm(ab2, cd2, 0x5410) ^ 0x80808080u;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 255u) | ((static_cast<uint32_t>(b) & 255u) << 8) |
         ((static_cast<uint32_t>(c) & 255u) << 16) | ((static_cast<uint32_t>(d) & 255u) << 24);
}

// One CTA per token. planes: [3*M][kp] int8, row 3t+p. Columns [K, kp) are 0.
// Requires kp % 16 == 0.
// The planes, exponent and non-finite flag of token row t (one CTA).
__device__ __forceinline__ void q8_planes_row(const float* __restrict__ x, long long ldx, int K, int kp,
                                              int8_t* __restrict__ planes, int* __restrict__ exps,
                                              int* __restrict__ nonfinite, int t, float* redf, int* redi) {
  const float* xr = x + static_cast<long long>(t) * ldx;
  const bool vec = ((K & 3) == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0);
  const int nchunk = (kp + 3) >> 2;  // 4-element chunks covering [0, kp)
  float4 reg[kPrepVec / 4];
  float amax = 0.f;
  int bad = 0;
  #pragma unroll
  for (int i = 0; i < kPrepVec / 4; ++i) {
    const int ch = threadIdx.x + i * blockDim.x;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ch < nchunk) {
      const int k = ch * 4;
      if (vec && k + 3 < K) {
        v = *reinterpret_cast<const float4*>(xr + k);
      } else {
        v.x = k < K ? xr[k] : 0.f;
        v.y = k + 1 < K ? xr[k + 1] : 0.f;
        v.z = k + 2 < K ? xr[k + 2] : 0.f;
        v.w = k + 3 < K ? xr[k + 3] : 0.f;
      }
    }
    reg[i] = v;
    bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  for (int ch = threadIdx.x + kPrepVec / 4 * blockDim.x; ch < nchunk; ch += blockDim.x) {
    for (int j = 0; j < 4; ++j) {
      const int k = ch * 4 + j;
      const float v = k < K ? xr[k] : 0.f;
      bad |= !isfinite(v);
      amax = fmaxf(amax, fabsf(v));
    }
  }
  block_max_or(amax, bad, redf, redi);
  int e = 0;
  if (!bad && amax > 0.f) {
    int E;
    frexpf(amax, &E);
    e = 22 - E;
  }
  uint32_t* p0 = reinterpret_cast<uint32_t*>(planes + static_cast<long long>(3 * t) * kp);
  uint32_t* p1 = reinterpret_cast<uint32_t*>(planes + static_cast<long long>(3 * t + 1) * kp);
  uint32_t* p2 = reinterpret_cast<uint32_t*>(planes + static_cast<long long>(3 * t + 2) * kp);
  #pragma unroll
  for (int i = 0; i < kPrepVec / 4; ++i) {
    const int ch = threadIdx.x + i * blockDim.x;
    if (ch < nchunk) {
      const float4 v = bad ? make_float4(0.f, 0.f, 0.f, 0.f) : reg[i];
      q8_digits4(v, e, p0[ch], p1[ch], p2[ch]);
    }
  }
  for (int ch = threadIdx.x + kPrepVec / 4 * blockDim.x; ch < nchunk; ch += blockDim.x) {
    int d[3][4];
    for (int j = 0; j < 4; ++j) {
      const int k = ch * 4 + j;
      const float v = (k < K && !bad) ? xr[k] : 0.f;
      q8_digits(v, e, d[0][j], d[1][j], d[2][j]);
    }
    p0[ch] = pack4(d[0][0], d[0][1], d[0][2], d[0][3]);
    p1[ch] = pack4(d[1][0], d[1][1], d[1][2], d[1][3]);
    p2[ch] = pack4(d[2][0], d[2][1], d[2][2], d[2][3]);
  }
  if (threadIdx.x == 0) {
    exps[t] = e;
    nonfinite[t] = bad;
  }
}

__global__ void __launch_bounds__(kPrepThreads) q8_planes_kernel(const float* __restrict__ x, long long ldx, int M,
                                                                 int K, int kp, int8_t* __restrict__ planes,
                                                                 int* __restrict__ exps, int* __restrict__ nonfinite) {
  pdl_launch_dependents();
  pdl_wait_prior();  // a programmatic dependent: the previous kernel may still read these outputs or write the inputs
  __shared__ float redf[32];
  __shared__ int redi[32];
  const int t = blockIdx.x;
  if (t >= M) return;
  q8_planes_row(x, ldx, K, kp, planes, exps, nonfinite, t, redf, redi);
}

// The planes of several independent activation matrices with the same token
// count in one launch: grid (M, count), problem blockIdx.y.
constexpr int kPlanesMaxGroup = 16;
struct PlanesProblem {
  const float* x;
  int8_t* planes;
  int* exps;
  int* nonfinite;
  int k, kp;
};
struct PlanesGroup {
  PlanesProblem prob[kPlanesMaxGroup];
  int count, m;
};

__global__ void __launch_bounds__(kPrepThreads) q8_planes_group_kernel(const __grid_constant__ PlanesGroup g) {
  pdl_launch_dependents();
  pdl_wait_prior();  // a programmatic dependent: the previous kernel may still read these outputs or write the inputs
  __shared__ float redf[32];
  __shared__ int redi[32];
  if (static_cast<int>(blockIdx.y) >= g.count || static_cast<int>(blockIdx.x) >= g.m) return;
  const PlanesProblem& pr = g.prob[blockIdx.y];
  q8_planes_row(pr.x, pr.k, pr.k, pr.kp, pr.planes, pr.exps, pr.nonfinite, blockIdx.x, redf, redi);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = (l < static_cast<int>(blockDim.x >> 5)) ? red[l] : 0.f;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// RMSNorm fused into the Q8 activation encoding (ops/src/kernels.rs:1346-1370,
// then the planes of q8_planes_kernel). Per row t of src: ss = sum_k src_k^2
// (f32, per-thread sums then a block tree; the reference sums sequentially),
// inv = 1 / sqrt(ss / K + eps), x_k = (src_k * inv) * g_k as the reference
// rounds them. The normalised rows go to xn ([M][K], for the exact recompute
// of rows holding NaN / Inf), then the digit planes, exponent and flag of x
// exactly as q8_planes_kernel makes them. One CTA per token.
__global__ void __launch_bounds__(kPrepThreads) q8_norm_planes_kernel(
    const float* __restrict__ src, long long lds, const float* __restrict__ g, float eps, int M, int K, int kp,
    float* __restrict__ xn, int8_t* __restrict__ planes, int* __restrict__ exps, int* __restrict__ nonfinite) {
  pdl_launch_dependents();
  pdl_wait_prior();  // a programmatic dependent: the previous kernel may still read these outputs or write the inputs
  __shared__ float redf[32];
  __shared__ int redi[32];
  const int t = blockIdx.x;
  if (t >= M) return;
  const float* sr = src + static_cast<long long>(t) * lds;
  float* xr = xn + static_cast<long long>(t) * K;
  float ss = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = sr[k];
    ss = __fadd_rn(ss, __fmul_rn(v, v));
  }
  ss = block_sum(ss, redf);
  const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps)));
  float amax = 0.f;
  int bad = 0;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float x = __fmul_rn(__fmul_rn(sr[k], inv), __ldg(g + k));
    xr[k] = x;
    bad |= !isfinite(x);
    amax = fmaxf(amax, fabsf(x));
  }
  block_max_or(amax, bad, redf, redi);  // (its barrier also makes xr visible to the whole CTA)
  int e = 0;
  if (!bad && amax > 0.f) {
    int E;
    frexpf(amax, &E);
    e = 22 - E;
  }
  uint32_t* p0 = reinterpret_cast<uint32_t*>(planes + static_cast<long long>(3 * t) * kp);
  uint32_t* p1 = reinterpret_cast<uint32_t*>(planes + static_cast<long long>(3 * t + 1) * kp);
  uint32_t* p2 = reinterpret_cast<uint32_t*>(planes + static_cast<long long>(3 * t + 2) * kp);
  const int nchunk = (kp + 3) >> 2;
  for (int ch = threadIdx.x; ch < nchunk; ch += blockDim.x) {
    int d[3][4];
    for (int j = 0; j < 4; ++j) {
      const int k = ch * 4 + j;
      const float v = (k < K && !bad) ? xr[k] : 0.f;
      q8_digits(v, e, d[0][j], d[1][j], d[2][j]);
    }
    p0[ch] = pack4(d[0][0], d[0][1], d[0][2], d[0][3]);
    p1[ch] = pack4(d[1][0], d[1][1], d[1][2], d[1][3]);
    p2[ch] = pack4(d[2][0], d[2][1], d[2][2], d[2][3]);
  }
  if (threadIdx.x == 0) {
    exps[t] = e;
    nonfinite[t] = bad;
  }
}

__device__ __forceinline__ uint16_t bf16_rn_bits(float v) {
  // Round to nearest even; a finite value that would round to infinity is
  // truncated instead so that hi stays finite and the residual stays exact.
  const uint32_t u = __float_as_uint(v);
  const uint32_t r = (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
  if ((r & 0x7f80u) == 0x7f80u) return static_cast<uint16_t>(u >> 16);
  return static_cast<uint16_t>(r);
}

__device__ __forceinline__ float bf16_val(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

// Three bf16 terms of one value; flags |= 2 / 4 for a non-zero mid / lo term,
// 256 for a non-finite value (which keeps only hi: NaN or +-Inf).
__device__ __forceinline__ void bf16_split(float v, uint16_t& h, uint16_t& m, uint16_t& l, int& flags) {
  if (!isfinite(v)) {
    flags |= 256;
    h = (v != v) ? 0x7fc0u : static_cast<uint16_t>(__float_as_uint(v) >> 16);
    m = 0;
    l = 0;
    return;
  }
  h = bf16_rn_bits(v);
  const float r1 = __fsub_rn(v, bf16_val(h));
  m = bf16_rn_bits(r1);
  const float r2 = __fsub_rn(r1, bf16_val(m));
  l = bf16_rn_bits(r2);
  if (m & 0x7fffu) flags |= 2;
  if (l & 0x7fffu) flags |= 4;
}

// Split terms for the normal-mode GEMM, layout out[t*3*kp + j*kp + k]. One
// CTA of kNormPrepThreads per token row. The hi plane is always written. The
// mid / lo plane of a row is written only when the row has non-zero values
// there now, or had them after the previous call (dirty[t] bits 2 / 4), so
// every plane keeps holding this call's exact terms while activations that
// are already bf16 values (the usual prefill input) cost one plane of writes.
// Rows with a non-zero mid / lo plane OR bit 2 / 4 into *orword; CTA 0 clears
// *orword_next for the next call (calls alternate between two words).
constexpr int kNormPrepThreads = 128;
constexpr int kNormPrepKeep = 8;  // float4 chunks per thread kept in registers

__device__ __forceinline__ uint2 pack_bf16x4(const uint16_t (&h)[4]) {
  return make_uint2(h[0] | (static_cast<uint32_t>(h[1]) << 16), h[2] | (static_cast<uint32_t>(h[3]) << 16));
}

// The split of one row (the body of the normal-mode prep kernels). kNf: also
// flag NaN / Inf (bit 256 of the row's flags; *nf = 1 for such a row, else 0)
// for the f32 GEMM, whose two split operands cannot carry them.
template <bool kNf>
__device__ __forceinline__ void norm_terms_row(const float* __restrict__ xr, int K, int kp, int vec,
                                               uint16_t* __restrict__ o0, uint8_t* __restrict__ dirty_t,
                                               int* __restrict__ nf_t, unsigned* __restrict__ orword, int* redi) {
  const int nchunk = kp >> 2;  // kp % 8 == 0
  const bool kept = nchunk <= kNormPrepKeep * kNormPrepThreads;
  const int old_dirty = *dirty_t;
  auto load = [&](int ch) -> float4 {
    const int k = ch * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ch < nchunk && k < K) {
      if (vec && k + 3 < K) {
        v = *reinterpret_cast<const float4*>(xr + k);
      } else {
        v.x = xr[k];
        v.y = k + 1 < K ? xr[k + 1] : 0.f;
        v.z = k + 2 < K ? xr[k + 2] : 0.f;
        v.w = k + 3 < K ? xr[k + 3] : 0.f;
      }
    }
    return v;
  };
  float4 keep[kNormPrepKeep];
  int flags = 0;
  // pass 1: hi plane and the row's term flags
  for (int c0 = 0; c0 < nchunk; c0 += kNormPrepKeep * kNormPrepThreads) {
    #pragma unroll
    for (int i = 0; i < kNormPrepKeep; ++i) keep[i] = load(c0 + threadIdx.x + i * kNormPrepThreads);
    #pragma unroll
    for (int i = 0; i < kNormPrepKeep; ++i) {
      const int ch = c0 + threadIdx.x + i * kNormPrepThreads;
      if (ch >= nchunk) break;
      const float4 v = keep[i];
      const uint32_t ux = __float_as_uint(v.x), uy = __float_as_uint(v.y);
      const uint32_t uz = __float_as_uint(v.z), uw = __float_as_uint(v.w);
      uint2 hi;
      if (((ux | uy | uz | uw) & 0xffffu) == 0u) {
        // already bf16 values (NaN and Inf included): hi is the top half
        hi = make_uint2((ux >> 16) | (uy & 0xffff0000u), (uz >> 16) | (uw & 0xffff0000u));
        if constexpr (kNf) {
          constexpr uint32_t E = 0x7f800000u;
          if ((ux & E) == E || (uy & E) == E || (uz & E) == E || (uw & E) == E) flags |= 256;
        }
      } else {
        uint16_t h[4], m[4], l[4];
        bf16_split(v.x, h[0], m[0], l[0], flags);
        bf16_split(v.y, h[1], m[1], l[1], flags);
        bf16_split(v.z, h[2], m[2], l[2], flags);
        bf16_split(v.w, h[3], m[3], l[3], flags);
        hi = pack_bf16x4(h);
      }
      reinterpret_cast<uint2*>(o0)[ch] = hi;
    }
  }
  flags = block_or(flags & (kNf ? (6 | 256) : 6), redi);
  const int need = (flags | old_dirty) & 6;
  // pass 2: mid / lo planes where needed
  if (need) {
    for (int c0 = 0; c0 < nchunk; c0 += kNormPrepKeep * kNormPrepThreads) {
      if (!kept) {
        #pragma unroll
        for (int i = 0; i < kNormPrepKeep; ++i) keep[i] = load(c0 + threadIdx.x + i * kNormPrepThreads);
      }
      #pragma unroll
      for (int i = 0; i < kNormPrepKeep; ++i) {
        const int ch = c0 + threadIdx.x + i * kNormPrepThreads;
        if (ch >= nchunk) break;
        int f = 0;
        uint16_t h[4], m[4], l[4];
        bf16_split(keep[i].x, h[0], m[0], l[0], f);
        bf16_split(keep[i].y, h[1], m[1], l[1], f);
        bf16_split(keep[i].z, h[2], m[2], l[2], f);
        bf16_split(keep[i].w, h[3], m[3], l[3], f);
        if (need & 2) reinterpret_cast<uint2*>(o0 + kp)[ch] = pack_bf16x4(m);
        if (need & 4) reinterpret_cast<uint2*>(o0 + 2 * kp)[ch] = pack_bf16x4(l);
      }
    }
  }
  if (threadIdx.x == 0) {
    if ((flags & 6) != old_dirty) *dirty_t = static_cast<uint8_t>(flags & 6);
    if constexpr (kNf) *nf_t = (flags & 256) ? 1 : 0;
    if (flags) atomicOr(orword, static_cast<unsigned>(flags));
  }
}

// zc != nullptr: also zero row t of C (zn columns, row stride ldc; zvec: rows
// 16-byte aligned), for a GEMM that adds partial sums into C.
__global__ void __launch_bounds__(kNormPrepThreads) bf16_terms_norm_kernel(
    const float* __restrict__ x, long long ldx, int M, int K, int kp, int vec, uint16_t* __restrict__ out,
    uint8_t* __restrict__ dirty, unsigned* __restrict__ orword, unsigned* __restrict__ orword_next,
    float* __restrict__ zc, long long ldc, int zn, int zvec) {
  pdl_launch_dependents();
  // Launched as a programmatic dependent of the previous kernel in the stream
  // (the GEMM of the previous call lets it start early): its term buffer,
  // flag words and C may still be in use until that kernel completes.
  pdl_wait_prior();
  __shared__ int redi[32];
  const int t = blockIdx.x;
  if (t >= M) return;
  if (t == 0 && threadIdx.x == 0) *orword_next = 0u;
  if (zc) {
    float* zr = zc + static_cast<long long>(t) * ldc;
    if (zvec) {
      for (int j = threadIdx.x; j < zn / 4; j += kNormPrepThreads)
        reinterpret_cast<float4*>(zr)[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = (zn / 4) * 4 + threadIdx.x; j < zn; j += kNormPrepThreads) zr[j] = 0.f;
    } else {
      for (int j = threadIdx.x; j < zn; j += kNormPrepThreads) zr[j] = 0.f;
    }
  }
  norm_terms_row<false>(x + static_cast<long long>(t) * ldx, K, kp, vec, out + static_cast<long long>(t) * 3 * kp,
                        dirty + t, nullptr, orword, redi);
}

// Split terms of both operands of the f32 GEMM C = A . B^T (A [M][K], B [N][K],
// row-major): CTA r < M splits row r of A, CTA M + r row r of B, into their
// own term buffers, dirty bits, non-finite flags and OR words (flag words as
// in bf16_terms_norm_kernel; CTA 0 clears both next words).
__global__ void __launch_bounds__(kNormPrepThreads) f32_terms_nt_kernel(
    const float* __restrict__ a, long long lda, int M, int vec_a, const float* __restrict__ b, long long ldb, int N,
    int vec_b, int K, int kp, uint16_t* __restrict__ ta, uint16_t* __restrict__ tb, uint8_t* __restrict__ dirty_a,
    uint8_t* __restrict__ dirty_b, int* __restrict__ nf_a, int* __restrict__ nf_b, unsigned* __restrict__ or_a,
    unsigned* __restrict__ or_a_next, unsigned* __restrict__ or_b, unsigned* __restrict__ or_b_next) {
  pdl_launch_dependents();
  pdl_wait_prior();  // a programmatic dependent: the previous kernel may still read these outputs or write the inputs
  __shared__ int redi[32];
  const int r = blockIdx.x;
  if (r == 0 && threadIdx.x == 0) {
    *or_a_next = 0u;
    *or_b_next = 0u;
  }
  if (r < M)
    norm_terms_row<true>(a + static_cast<long long>(r) * lda, K, kp, vec_a, ta + static_cast<long long>(r) * 3 * kp,
                         dirty_a + r, nf_a + r, or_a, redi);
  else if (r - M < N)
    norm_terms_row<true>(b + static_cast<long long>(r - M) * ldb, K, kp, vec_b,
                         tb + static_cast<long long>(r - M) * 3 * kp, dirty_b + (r - M), nf_b + (r - M), or_b, redi);
}

// Split terms of both operands of the NN f32 GEMM C = A . B (A [M][K], B
// [K][N], row-major) in one launch of kNormPrepThreads-thread CTAs.
//  - CTAs [0, ntx * nty) split B transposed: out_b[n*3*kp + j*kp + k],
//    columns [K, kp) zero, kp % 64 == 0; CTA (tx, ty) takes the 64 (k) x 64
//    (n) tile (ty, tx) through shared memory (loads coalesced along n, stores
//    along k). nf_b[n] becomes 1 for a column holding NaN / Inf (nf_b is
//    cleared by the previous NN call; CTAs with ty == 0 clear their columns of
//    nf_b_next for the next one); the tiles OR their term flags into *or_b.
//  - CTAs [ntx * nty, + M) split the rows of A as f32_terms_nt_kernel does.
// CTA 0 clears both next flag words.
constexpr int kTransTile = 64;
__global__ void __launch_bounds__(kNormPrepThreads) f32_terms_nn_kernel(
    const float* __restrict__ a, long long lda, int M, int vec_a, const float* __restrict__ b, long long ldb, int N,
    int K, int kp, int ntx, int nty, uint16_t* __restrict__ ta, uint16_t* __restrict__ tb,
    uint8_t* __restrict__ dirty_a, int* __restrict__ nf_a, int* __restrict__ nf_b, int* __restrict__ nf_b_next,
    unsigned* __restrict__ or_a, unsigned* __restrict__ or_a_next, unsigned* __restrict__ or_b,
    unsigned* __restrict__ or_b_next) {
  pdl_launch_dependents();
  pdl_wait_prior();  // a programmatic dependent: the previous kernel may still read these outputs or write the inputs
  __shared__ float tile[kTransTile][kTransTile + 1];
  __shared__ int redi[32];
  const int cta = blockIdx.x;
  if (cta == 0 && threadIdx.x == 0) {
    *or_a_next = 0u;
    *or_b_next = 0u;
  }
  if (cta >= ntx * nty) {
    const int r = cta - ntx * nty;
    if (r < M)
      norm_terms_row<true>(a + static_cast<long long>(r) * lda, K, kp, vec_a, ta + static_cast<long long>(r) * 3 * kp,
                           dirty_a + r, nf_a + r, or_a, redi);
    return;
  }
  const int tx = cta % ntx, ty = cta / ntx;
  const int n0 = tx * kTransTile, k0 = ty * kTransTile;
  if (ty == 0 && threadIdx.x < kTransTile && n0 + static_cast<int>(threadIdx.x) < N) nf_b_next[n0 + threadIdx.x] = 0;
  for (int i = threadIdx.x; i < kTransTile * kTransTile; i += kNormPrepThreads) {
    const int kk = i / kTransTile, nn = i - kk * kTransTile;
    const int k = k0 + kk, n = n0 + nn;
    tile[kk][nn] = (k < K && n < N) ? b[static_cast<long long>(k) * ldb + n] : 0.f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int my_flags = 0;
  for (int nn = warp; nn < kTransTile; nn += kNormPrepThreads / 32) {
    const int n = n0 + nn;
    if (n >= N) break;
    int f = 0;
    uint16_t h0, m0, l0, h1, m1, l1;
    bf16_split(tile[2 * lane][nn], h0, m0, l0, f);
    bf16_split(tile[2 * lane + 1][nn], h1, m1, l1, f);
    uint32_t* o = reinterpret_cast<uint32_t*>(tb + static_cast<long long>(n) * 3 * kp + k0) + lane;
    o[0] = h0 | (static_cast<uint32_t>(h1) << 16);
    o[kp / 2] = m0 | (static_cast<uint32_t>(m1) << 16);
    o[kp] = l0 | (static_cast<uint32_t>(l1) << 16);
    f = warp_or(f);
    if (lane == 0 && (f & 256)) atomicOr(nf_b + n, 1);
    my_flags |= f;
  }
  my_flags = block_or(my_flags, redi);
  if (threadIdx.x == 0 && my_flags) atomicOr(or_b, static_cast<unsigned>(my_flags));
}

// One CTA per token. Layout 0 (swap): out[(3t+j)*kp + k]. Layout 1 (normal):
// out[t*3*kp + j*kp + k]. Columns [K, kp) are 0; kp % 8 == 0. term_flags[t]
// gets 1 | (2 if a mid term is non-zero) | (4 if a lo term is non-zero). The
// last CTA to finish (counted on done[0], which it resets) ORs all rows into
// done[1], so a consumer reads one word instead of M.
__global__ void __launch_bounds__(kPrepThreads) bf16_terms_kernel(const float* __restrict__ x, long long ldx, int M,
                                                                  int K, int kp, int layout,
                                                                  uint16_t* __restrict__ out,
                                                                  int* __restrict__ term_flags,
                                                                  int* __restrict__ nonfinite,
                                                                  unsigned* __restrict__ done) {
  pdl_launch_dependents();
  pdl_wait_prior();  // a programmatic dependent: the previous kernel may still read these outputs or write the inputs
  __shared__ int redi[32];
  __shared__ int is_last;
  const int t = blockIdx.x;
  if (t >= M) return;
  const float* xr = x + static_cast<long long>(t) * ldx;
  const bool vec = ((K & 3) == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0);
  uint16_t* o0 = layout == 0 ? out + static_cast<long long>(3 * t) * kp : out + static_cast<long long>(t) * 3 * kp;
  uint16_t* o1 = o0 + kp;
  uint16_t* o2 = o1 + kp;
  const int nchunk = kp >> 2;  // kp % 8 == 0
  int flags = 0;
  for (int ch = threadIdx.x; ch < nchunk; ch += blockDim.x) {
    const int k = ch * 4;
    float4 v;
    if (vec && k + 3 < K) {
      v = *reinterpret_cast<const float4*>(xr + k);
    } else {
      v.x = k < K ? xr[k] : 0.f;
      v.y = k + 1 < K ? xr[k + 1] : 0.f;
      v.z = k + 2 < K ? xr[k + 2] : 0.f;
      v.w = k + 3 < K ? xr[k + 3] : 0.f;
    }
    uint16_t h[4], m[4], l[4];
    bf16_split(v.x, h[0], m[0], l[0], flags);
    bf16_split(v.y, h[1], m[1], l[1], flags);
    bf16_split(v.z, h[2], m[2], l[2], flags);
    bf16_split(v.w, h[3], m[3], l[3], flags);
    reinterpret_cast<uint2*>(o0)[ch] = make_uint2(h[0] | (static_cast<uint32_t>(h[1]) << 16),
                                                  h[2] | (static_cast<uint32_t>(h[3]) << 16));
    reinterpret_cast<uint2*>(o1)[ch] = make_uint2(m[0] | (static_cast<uint32_t>(m[1]) << 16),
                                                  m[2] | (static_cast<uint32_t>(m[3]) << 16));
    reinterpret_cast<uint2*>(o2)[ch] = make_uint2(l[0] | (static_cast<uint32_t>(l[1]) << 16),
                                                  l[2] | (static_cast<uint32_t>(l[3]) << 16));
  }
  flags = block_or(flags, redi);
  if (threadIdx.x == 0) {
    term_flags[t] = (flags & 6) | 1;
    nonfinite[t] = (flags >> 8) & 1;
    // release this row's flags; the last CTA's acquire sees every row's
    is_last = (atom_add_acq_rel_gpu(done, 1u) == static_cast<unsigned>(M - 1));
  }
  __syncthreads();
  if (is_last) {
    int orv = 0;
    for (int i = threadIdx.x; i < M; i += blockDim.x) orv |= __ldcg(term_flags + i);
    orv = block_or(orv, redi);
    if (threadIdx.x == 0) {
      done[1] = static_cast<unsigned>(orv);
      done[0] = 0u;
    }
  }
}

// ----------------------------------------------------- CUDA-core fallbacks
// One warp per output (t, n). Used only when the operands cannot be fed to TMA
// (row pitch not a multiple of 16 bytes or unaligned base pointers).

// Q8 from the digit planes, exactly as the tensor-core path combines them.
__global__ void q8_generic_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                  const int8_t* __restrict__ planes, int kp, const int* __restrict__ exps,
                                  const int* __restrict__ nonfinite, const float* __restrict__ x, long long ldx,
                                  float* __restrict__ c, long long ldc, int M, int N, int K) {
  pdl_wait_prior();
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<long long>(M) * N) return;
  const int t = static_cast<int>(gw / N), n = static_cast<int>(gw % N);
  const int8_t* qr = q + static_cast<long long>(n) * K;
  float out;
  if (nonfinite[t]) {
    // sequential f32, same NaN/Inf classification as the reference
    float s = 0.f;
    if (lane == 0) {
      const float* xr = x + static_cast<long long>(t) * ldx;
      for (int k = 0; k < K; ++k) s = __fadd_rn(s, __fmul_rn(xr[k], static_cast<float>(qr[k])));
    }
    out = __fmul_rn(s, scale[n]);
  } else {
    const int8_t* p0 = planes + static_cast<long long>(3 * t) * kp;
    long long a0 = 0, a1 = 0, a2 = 0;
    for (int k = lane; k < K; k += 32) {
      const int w = qr[k];
      a0 += w * p0[k];
      a1 += w * p0[kp + k];
      a2 += w * p0[2 * kp + k];
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a0 += __shfl_xor_sync(0xffffffffu, a0, o);
      a1 += __shfl_xor_sync(0xffffffffu, a1, o);
      a2 += __shfl_xor_sync(0xffffffffu, a2, o);
    }
    const long long v = a2 * 65536ll + a1 * 256ll + a0;
    out = __fmul_rn(__double2float_rn(ldexp(static_cast<double>(v), -exps[t])), scale[n]);
  }
  if (lane == 0) c[static_cast<long long>(t) * ldc + n] = out;
}

// bf16 weights: f32 FMA dot product, warp tree reduction.
__global__ void bf16_generic_kernel(const uint16_t* __restrict__ b, const float* __restrict__ x, long long ldx,
                                    float* __restrict__ c, long long ldc, int M, int N, int K) {
  pdl_wait_prior();
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<long long>(M) * N) return;
  const int t = static_cast<int>(gw / N), n = static_cast<int>(gw % N);
  const uint16_t* br = b + static_cast<long long>(n) * K;
  const float* xr = x + static_cast<long long>(t) * ldx;
  float s = 0.f;
  for (int k = lane; k < K; k += 32) s = __fmaf_rn(xr[k], bf16_val(br[k]), s);
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  if (lane == 0) c[static_cast<long long>(t) * ldc + n] = s;
}

// int8 x int8 -> int32, then f32(acc)*scale. Exact.
__global__ void i8i8_generic_kernel(const int8_t* __restrict__ xq, const int8_t* __restrict__ w,
                                    const float* __restrict__ scale, float* __restrict__ c,
                                    int32_t* __restrict__ acc_out, int M, int N, int K) {
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<long long>(M) * N) return;
  const int m = static_cast<int>(gw / N), n = static_cast<int>(gw % N);
  const int8_t* xr = xq + static_cast<long long>(m) * K;
  const int8_t* wr = w + static_cast<long long>(n) * K;
  int a = 0;
  for (int k = lane; k < K; k += 32) a += static_cast<int>(xr[k]) * static_cast<int>(wr[k]);
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  if (lane == 0) {
    const long long idx = static_cast<long long>(m) * N + n;
    if (acc_out) acc_out[idx] = a;
    if (c) c[idx] = __fmul_rn(__int2float_rn(a), scale[n]);
  }
}

}  // namespace vmlm
