#pragma once

// Greedy sampling: the index of the largest logit, the lowest index among equal values (as
// torch.argmax), in two launches — the drop-in for the reference's kernels/argmax.hpp (interface
// :35-42, :44-70; launched by src/engine/model.hip:96-100 with n_parts blocks, then one block).
// Stage 1: block b scans the contiguous range [b * per, (b + 1) * per) and writes its best
// (value, index); stage 2: one block reduces the partials. Both reduce with warp shuffles under
// the order (greater value, then lower index).

#include <cuda_runtime.h>

#include "wave.hpp"

namespace miso::kernels {

struct ArgmaxParams {
  const float* x;
  unsigned n;
  float* part_v;  // [gridDim.x of stage 1]
  int* part_i;
  unsigned n_parts;
  int* out;  // [1]
};

namespace argmax_detail {

__device__ __forceinline__ void better(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i))
    v = ov, i = oi;
}

// (value, index) reduction over the block; thread 0 gets the result.
template <int kBlock>
__device__ inline void block_argmax(float& v, int& i) {
  __shared__ float sv[kBlock / kWave];
  __shared__ int si[kBlock / kWave];
#pragma unroll
  for (int off = kWave / 2; off > 0; off >>= 1)
    better(v, i, __shfl_xor_sync(0xffffffffu, v, off), __shfl_xor_sync(0xffffffffu, i, off));
  if (threadIdx.x % kWave == 0)
    sv[threadIdx.x / kWave] = v, si[threadIdx.x / kWave] = i;
  __syncthreads();
  if (threadIdx.x == 0)
    for (int w = 1; w < kBlock / kWave; ++w)
      better(v, i, sv[w], si[w]);
  __syncthreads();
}

}  // namespace argmax_detail

template <int kBlock>
__global__ void __launch_bounds__(kBlock) argmax_partial_kernel(ArgmaxParams p) {
  const unsigned per = (p.n + gridDim.x - 1) / gridDim.x;
  const unsigned lo = blockIdx.x * per, hi = min(p.n, lo + per);
  float v = -INFINITY;
  int idx = 0x7FFFFFFF;
  for (unsigned j = lo + threadIdx.x; j < hi; j += kBlock)
    argmax_detail::better(v, idx, p.x[j], static_cast<int>(j));
  argmax_detail::block_argmax<kBlock>(v, idx);
  if (threadIdx.x == 0)
    p.part_v[blockIdx.x] = v, p.part_i[blockIdx.x] = idx;
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) argmax_final_kernel(ArgmaxParams p) {
  float v = -INFINITY;
  int idx = 0x7FFFFFFF;
  for (unsigned j = threadIdx.x; j < p.n_parts; j += kBlock)
    argmax_detail::better(v, idx, p.part_v[j], p.part_i[j]);
  argmax_detail::block_argmax<kBlock>(v, idx);
  if (threadIdx.x == 0)
    *p.out = idx;
}

}  // namespace miso::kernels
