// probe.cuh -- tensor-core throughput probe (diagnostics, vmlm_probe_mma_peak).
//
// One CTA per SM issues back-to-back tcgen05.mma instructions of the largest
// single-CTA shape (M = 128, N = 256, one 128-byte K slice of each operand per
// four instructions) on operands that stay in shared memory, so nothing but
// the tensor pipe is timed. The operands hold pseudo-random data (the pipe's
// power draw, and so the clock under the power cap, depends on it). The
// measured rate is the dense peak the GEMM kernels of this library are
// compared against: kind::i8 for the int8 x int8 GEMM, kind::f16 (bf16
// operands) to check the probe against the cuBLAS bf16 figure.
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace vmlm {

constexpr int kProbeThreads = 128;
constexpr uint32_t kProbeAccCols = 256;   // one 128 x 256 accumulator (f32 / s32)
constexpr uint32_t kProbeABytes = 128 * 128;  // A: 128 rows x 128 bytes (one swizzle atom wide)
constexpr uint32_t kProbeBBytes = 256 * 128;  // B: 256 rows x 128 bytes
constexpr uint32_t kProbeSmem = 1024 + kProbeABytes + kProbeBBytes;
// Upper bound on the loop count, so that even at a quarter of the expected
// rate the probe ends well inside the 1 s bounded wait.
constexpr int kProbeMaxIters = 200000;

// KIND 0: kind::f16 with bf16 operands, f32 accumulate (K = 16 per instruction).
// KIND 1: kind::i8 with signed 8-bit operands, s32 accumulate (K = 32).
// Each instruction covers 32 bytes of K; four cover the 128-byte slice, whose
// descriptors start 32 bytes apart inside the 128-byte swizzle atom.
template <int KIND>
__global__ void __launch_bounds__(kProbeThreads, 1) mma_peak_kernel(int iters, int* err) {
  extern __shared__ uint8_t probe_raw[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(probe_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = base;
  uint8_t* sb = base + kProbeABytes;
  // pseudo-random operands: bf16 values of magnitude in [1, 2) with random
  // signs (no NaN / Inf), or arbitrary signed bytes
  for (uint32_t i = threadIdx.x; i < (kProbeABytes + kProbeBBytes) / 4; i += kProbeThreads) {
    uint32_t h = (i + 1u) * 2654435761u ^ (blockIdx.x * 40503u);
    h ^= h >> 13;
    h *= 0x5bd1e995u;
    h ^= h >> 15;
    uint32_t v = h;
    if (KIND == 0) v = (h & 0x807F807Fu) | 0x3F803F80u;
    reinterpret_cast<uint32_t*>(base)[i] = v;
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x < 32) tmem_alloc(&tmem_slot, kProbeAccCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = KIND == 0 ? umma_idesc(1, 1, 128, 256) : umma_idesc(2, 1, 128, 256);
    const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb);
    #pragma unroll 1
    for (int it = 0; it < iters; ++it) {
      #pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = umma_desc_sw128(a0 + 32u * kk);
        const uint64_t bd = umma_desc_sw128(b0 + 32u * kk);
        if (KIND == 0)
          umma_f16(tmem, ad, bd, idesc, (it | kk) ? 1u : 0u);
        else
          umma_i8(tmem, ad, bd, idesc, (it | kk) ? 1u : 0u);
      }
    }
    umma_commit(&bar);
    // a long loop: the bounded wait allows the whole probe (iters is capped on the host)
    mbar_wait(&bar, 0, err, &abort_flag, kDevTimeoutFull, false);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem, kProbeAccCols);
}

}  // namespace vmlm
