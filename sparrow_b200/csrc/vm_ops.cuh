// vm_ops.cuh -- the VM ops next to the quantised linear layer in a decode step
// (OP_GEMV, OP_EMB), as CUDA-core kernels: each streams its operand once from
// HBM and has no tensor-core shape.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace vmlm {

// Device error codes of OP_EMB (the VM prints the message and exits 9).
constexpr int kDevEmbRange = 101;     // "EMB: row index out of range"
constexpr int kDevEmbFraction = 102;  // "EMB: row index is not an integer"

// OP_GEMV (core/src/interp.rs:815-827): c[i] = sum_p a[i * k + p] * b[p], a
// [m, k] row-major. One warp per row: float4 loads when a's rows and b are
// 16-byte aligned, a partial sum per lane, then a warp tree (f32; the
// reference sums each row sequentially).
constexpr int kGemvWarps = 8;

__global__ void __launch_bounds__(kGemvWarps * 32) gemv_f32_kernel(const float* __restrict__ a,
                                                                   const float* __restrict__ b, float* __restrict__ c,
                                                                   int m, int k, int vec) {
  pdl_launch_dependents();
  const int row = blockIdx.x * kGemvWarps + static_cast<int>(threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= m) return;
  const float* ar = a + static_cast<long long>(row) * k;
  float s = 0.f;
  int p0 = 0;
  if (vec) {
    const int k4 = k & ~3;
    for (int p = lane * 4; p < k4; p += 128) {
      const float4 va = *reinterpret_cast<const float4*>(ar + p);
      const float4 vb = __ldg(reinterpret_cast<const float4*>(b + p));
      s = fmaf(va.x, vb.x, s);
      s = fmaf(va.y, vb.y, s);
      s = fmaf(va.z, vb.z, s);
      s = fmaf(va.w, vb.w, s);
    }
    p0 = k4;
  }
  for (int p = p0 + lane; p < k; p += 32) s = fmaf(ar[p], __ldg(b + p), s);
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) c[row] = s;
}

// OP_EMB (core/src/interp.rs:1351-1420) for m rows at once: out[t][:] =
// f32(table[r][:]) with r = idx[t], an f32 that must be an integer in
// [0, rows). dtype 4: bf16 table (widened exactly, (u32)h << 16); 0: f32. A
// bad index writes nothing for its row and records kDevEmbRange /
// kDevEmbFraction in *err, where the VM prints and exits 9. Grid (m, column
// blocks of 1024).
__global__ void __launch_bounds__(256) emb_kernel(const void* __restrict__ table, int dtype, long long rows, int cols,
                                                  const float* __restrict__ idx, int m, float* __restrict__ out,
                                                  int* __restrict__ err) {
  const int t = blockIdx.x;
  if (t >= m) return;
  const float rowf = __ldg(idx + t);
  if (!(rowf >= 0.f) || rowf >= static_cast<float>(rows)) {  // NaN fails every ordered comparison
    if (threadIdx.x == 0) atomicCAS(err, 0, kDevEmbRange);
    return;
  }
  const long long r = static_cast<long long>(rowf);
  if (static_cast<float>(r) != rowf) {
    if (threadIdx.x == 0) atomicCAS(err, 0, kDevEmbFraction);
    return;
  }
  float* o = out + static_cast<long long>(t) * cols;
  const int c0 = blockIdx.y * 1024;
  const int c1 = c0 + 1024 < cols ? c0 + 1024 : cols;
  if (dtype == 4) {
    const uint16_t* src = static_cast<const uint16_t*>(table) + r * cols;
    for (int i = c0 + static_cast<int>(threadIdx.x); i < c1; i += blockDim.x)
      o[i] = __uint_as_float(static_cast<uint32_t>(__ldg(src + i)) << 16);
  } else {
    const float* src = static_cast<const float*>(table) + r * cols;
    for (int i = c0 + static_cast<int>(threadIdx.x); i < c1; i += blockDim.x) o[i] = __ldg(src + i);
  }
}

}  // namespace vmlm
