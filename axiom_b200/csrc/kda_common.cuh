// Shared device helpers of the KDA library: element loads/stores for the two
// supported element types and small launch utilities.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "kda_b200.h"

namespace kda {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const bf16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void stf(float* p, float x) { *p = x; }
__device__ __forceinline__ void stf(bf16* p, float x) { *p = __float2bfloat16_rn(x); }

// Convert a status of the CUDA runtime after a launch into a KDA status.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Opt a kernel into more than 48 KB of dynamic shared memory, once per device.
template <typename Kern>
// The flags are atomics: host threads may launch concurrently (the calls are
// reentrant); setting the attribute twice is harmless, so a plain test-and-set
// suffices.
inline int ensure_smem(Kern kern, int bytes, std::atomic<bool>* done_per_device, int max_devices = 64) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= max_devices) return KDA_ERR_DEVICE;
  if (!done_per_device[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
      return KDA_ERR_LAUNCH;
    done_per_device[dev].store(true, std::memory_order_release);
  }
  return KDA_OK;
}

// Column sums over the 32 lanes of a warp: every lane holds N consecutive
// columns v[0..N-1] (N a power of two, 2 <= N <= 32); the result, on every lane, is column
// (lane % N) summed over all 32 lanes.  Halving exchanges (N/2 + ... + 1
// shuffles) leave lane l with column l % N summed over its group of N lanes;
// log2(32 / N) more shuffles add the groups.
template <int N>
__device__ __forceinline__ float warp_colsum(float (&v)[N], int lane) {
#pragma unroll
  for (int off = N / 2; off >= 1; off >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int j = 0; j < off; ++j) {
      const float send = up ? v[j] : v[j + off];
      const float recv = __shfl_xor_sync(0xffffffffu, send, off);
      v[j] = (up ? v[j + off] : v[j]) + recv;
    }
  }
  float s = v[0];
#pragma unroll
  for (int off = N; off < 32; off <<= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  return s;
}

}  // namespace kda
