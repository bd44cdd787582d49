// Shared helpers for the sm_100a kernels of the beam-search decode path.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/grs_b200.h"

#define GRS_CUDA_CHECK_LAUNCH()                                   \
  do {                                                            \
    cudaError_t _e = cudaGetLastError();                          \
    if (_e != cudaSuccess) return GRS_ERR_CUDA;                   \
  } while (0)

namespace grs {

// Every kernel launch of the library passes its stream through counted(),
// which bumps the process-wide launch counter read by grs_launch_count().
void note_launch();
inline cudaStream_t counted(cudaStream_t stream) {
  note_launch();
  return stream;
}

// Element loads/stores for the two arena dtypes: bf16 (device arenas) and
// fp32 (the CPU-equivalence configuration run on the GPU).
__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Record the first error of a launch in a device status word (0 = ok).
__device__ __forceinline__ void set_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// splitmix64 finaliser (Steele, Lea & Flood 2014; constants from Vigna's
// published reference).  Used for order-independent topology fingerprints.
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t node_component(int64_t slot, int64_t gate) {
  return mix64((1ull << 62) | ((uint64_t)slot << 16) | ((uint64_t)gate & 0xffffull));
}
__host__ __device__ __forceinline__ uint64_t edge_component(int64_t src, int64_t dst,
                                                            int64_t sp, int64_t dp) {
  return mix64((2ull << 62) | ((uint64_t)src << 36) | ((uint64_t)dst << 12) |
               (((uint64_t)sp & 63ull) << 6) | ((uint64_t)dp & 63ull));
}

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

}  // namespace grs
