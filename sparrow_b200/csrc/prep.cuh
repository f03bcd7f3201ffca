// prep.cuh -- activation preparation kernels and CUDA-core kernels for shapes
// the TMA path cannot take (K not a multiple of 16 bytes, unaligned rows).
//
// Q8 activations are encoded as three signed 8-bit digit planes per token:
//   e   = 22 - E  where max|x_t| = f * 2^E, f in [0.5, 1)   (e = 0 for a zero row)
//   X   = rint(x * 2^e)              |X| <= 2^22, exact scaling in f64
//   X   = d0 + 256*d1 + 65536*d2     d0, d1 in [-128,127], d2 in [-64,64]
// so sum_k x_k*q_k = 2^-e * sum_p 256^p * (sum_k d_p,k * q_k) up to the
// 2^-23*max|x| rounding of X; the three int32 sums are exact.
//
// bf16 activations (f32 in, bf16 weights) are split into three bf16 terms
//   hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)
// (each difference is exact in f32), which carry 24 significant bits.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace vmlm {

constexpr int kPrepThreads = 256;

__device__ __forceinline__ float block_max(float v, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (blockDim.x >> 5)) ? red[l] : 0.f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ int block_or(int v, int* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (blockDim.x >> 5)) ? red[l] : 0;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// One CTA per token. planes: [3*M][kp] int8, row 3t+p. Columns [K, kp) are 0.
__global__ void __launch_bounds__(kPrepThreads) q8_planes_kernel(const float* __restrict__ x, long long ldx, int M,
                                                                 int K, int kp, int8_t* __restrict__ planes,
                                                                 int* __restrict__ exps, int* __restrict__ nonfinite) {
  pdl_launch_dependents();
  __shared__ float redf[32];
  __shared__ int redi[32];
  const int t = blockIdx.x;
  if (t >= M) return;
  const float* xr = x + static_cast<long long>(t) * ldx;
  float amax = 0.f;
  int bad = 0;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = xr[k];
    if (!isfinite(v))
      bad = 1;
    else
      amax = fmaxf(amax, fabsf(v));
  }
  amax = block_max(amax, redf);
  bad = block_or(bad, redi);
  int e = 0;
  if (!bad && amax > 0.f) {
    int E;
    frexpf(amax, &E);
    e = 22 - E;
  }
  int8_t* p0 = planes + static_cast<long long>(3 * t) * kp;
  int8_t* p1 = p0 + kp;
  int8_t* p2 = p1 + kp;
  for (int k = threadIdx.x; k < kp; k += blockDim.x) {
    int X = 0;
    if (k < K && !bad) X = __double2int_rn(ldexp(static_cast<double>(xr[k]), e));
    const int d0 = ((X + 128) & 255) - 128;
    const int X1 = (X - d0) >> 8;
    const int d1 = ((X1 + 128) & 255) - 128;
    const int d2 = (X1 - d1) >> 8;
    p0[k] = static_cast<int8_t>(d0);
    p1[k] = static_cast<int8_t>(d1);
    p2[k] = static_cast<int8_t>(d2);
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

// One CTA per token. Layout 0 (swap): out[(3t+j)*kp + k]. Layout 1 (normal):
// out[t*3*kp + j*kp + k]. Columns [K, kp) are 0. term_flags[t] |= 1<<j for
// every term j that is non-zero somewhere in the row. The last CTA to finish
// (counted on done[0], which it resets) ORs all rows into done[1], so a
// consumer reads one word instead of M.
__global__ void __launch_bounds__(kPrepThreads) bf16_terms_kernel(const float* __restrict__ x, long long ldx, int M,
                                                                  int K, int kp, int layout,
                                                                  uint16_t* __restrict__ out,
                                                                  int* __restrict__ term_flags,
                                                                  int* __restrict__ nonfinite,
                                                                  unsigned* __restrict__ done) {
  pdl_launch_dependents();
  __shared__ int redi[32];
  __shared__ int is_last;
  const int t = blockIdx.x;
  if (t >= M) return;
  const float* xr = x + static_cast<long long>(t) * ldx;
  uint16_t* o0 = layout == 0 ? out + static_cast<long long>(3 * t) * kp : out + static_cast<long long>(t) * 3 * kp;
  uint16_t* o1 = o0 + kp;
  uint16_t* o2 = o1 + kp;
  int flags = 0, bad = 0;
  for (int k = threadIdx.x; k < kp; k += blockDim.x) {
    uint16_t h = 0, m = 0, l = 0;
    if (k < K) {
      const float v = xr[k];
      if (!isfinite(v)) {
        bad = 1;
        h = static_cast<uint16_t>(__float_as_uint(v) >> 16);
        if (v != v) h = 0x7fc0u;
      } else {
        h = bf16_rn_bits(v);
        const float r1 = __fsub_rn(v, bf16_val(h));
        m = bf16_rn_bits(r1);
        const float r2 = __fsub_rn(r1, bf16_val(m));
        l = bf16_rn_bits(r2);
      }
    }
    o0[k] = h;
    o1[k] = m;
    o2[k] = l;
    if (m & 0x7fffu) flags |= 2;
    if (l & 0x7fffu) flags |= 4;
  }
  flags = block_or(flags, redi);
  bad = block_or(bad, redi);
  if (threadIdx.x == 0) {
    term_flags[t] = flags | 1;
    nonfinite[t] = bad;
    __threadfence();
    is_last = (atomicAdd(done, 1u) == static_cast<unsigned>(M - 1));
  }
  __syncthreads();
  if (is_last) {
    __threadfence();
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
    int a0 = 0, a1 = 0, a2 = 0;
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
    const long long v = static_cast<long long>(a2) * 65536ll + static_cast<long long>(a1) * 256ll + a0;
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
