#pragma once

// Warp and block reductions for the drop-in kernels (reference interface: kernels/wave.hpp:9-64).
//
// CUDA warps are 32 lanes wide, so kWave is 32 here (the gfx906 reference uses 64-lane
// wavefronts). The block_* functions keep the reference meaning — a reduction over the whole
// block, returned to every thread — and need kBlock / kWave floats of shared scratch.
// wave_sum / wave_max return the reduction in every lane (a butterfly), which is a superset of
// the reference's "valid in the last lane".

#include <cuda_runtime.h>

namespace miso::kernels {

constexpr int kWave = 32;

template <class Op>
__device__ __forceinline__ float wave_reduce(float v, Op op) {
#pragma unroll
  for (int off = kWave / 2; off > 0; off >>= 1)
    v = op(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ float wave_sum(float v) {
  return wave_reduce(v, [](float a, float b) { return a + b; });
}

__device__ __forceinline__ float wave_max(float v) {
  return wave_reduce(v, [](float a, float b) { return fmaxf(a, b); });
}

// Reduction over a block of kBlock threads; every thread gets the result. Two barriers.
template <int kBlock, class Op>
__device__ __forceinline__ float block_reduce(float v, float* scratch, Op op) {
  static_assert(kBlock % kWave == 0, "block must be whole warps");
  v = wave_reduce(v, op);
  if (threadIdx.x % kWave == 0)
    scratch[threadIdx.x / kWave] = v;
  __syncthreads();
  float r = scratch[0];
#pragma unroll
  for (int w = 1; w < kBlock / kWave; ++w)
    r = op(r, scratch[w]);
  __syncthreads();
  return r;
}

template <int kBlock>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  return block_reduce<kBlock>(v, scratch, [](float a, float b) { return a + b; });
}

template <int kBlock>
__device__ __forceinline__ float block_max(float v, float* scratch) {
  return block_reduce<kBlock>(v, scratch, [](float a, float b) { return fmaxf(a, b); });
}

}  // namespace miso::kernels
