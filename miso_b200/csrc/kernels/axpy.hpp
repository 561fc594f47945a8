#pragma once

// y = a * x + y, the smallest operator of the reference's operator pattern (kernels/axpy.hpp:
// 12-31): a __device__ body over an explicit range of work items [first, first + count) and a
// grid-stride __global__ wrapper, so the body can also run inside a persistent kernel. The
// multiply and the add round separately (no contraction), as on a CPU without FMA.

#include <cuda_runtime.h>

namespace miso::kernels {

struct AxpyParams {
  float a;
  const float* x;
  float* y;
  unsigned n;
};

// Work items [first, first + count); one work item is one element.
template <int kBlock>
__device__ inline void axpy_op(const AxpyParams& p, unsigned first, unsigned count) {
  const unsigned end = first + count;
  for (unsigned i = first + blockIdx.x * kBlock + threadIdx.x; i < end; i += gridDim.x * kBlock)
    p.y[i] = __fadd_rn(__fmul_rn(p.a, p.x[i]), p.y[i]);
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) axpy_kernel(AxpyParams p) {
  axpy_op<kBlock>(p, 0, p.n);
}

}  // namespace miso::kernels
