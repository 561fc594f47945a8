// Test support (not product code): every instantiation of the drop-in attn_combine templates
// plus an independent serial combine, so the GPU tests can check the reference's bit-exactness
// contract for the combine (tests/test_attn_splitk.hip:21-96 of penta2himajin/miso): every
// variant must produce exactly the bits of a plain serial FP32 merge compiled by the same nvcc.

#include <cuda_runtime.h>

#include "kernels/attention_decode.hpp"

namespace k = miso::kernels;

namespace {

// Serial FP32 merge, one thread per (head, dim): M = max, then L += w * l and o += w * o_c in
// split order with w = __expf(m - M); core = o / L / (1 + __expf(-gate)). Writes only the
// 64-wide dimension tiles in [first_tile, first_tile + n_tiles).
__global__ void combine_serial(k::AttnCombineParams p, unsigned first_tile, unsigned n_tiles) {
  constexpr unsigned kDim = 256, kGroup = 8;
  const unsigned h = blockIdx.x, d = threadIdx.x;
  const unsigned kvh = h / kGroup, hl = h % kGroup;
  float M = -__int_as_float(0x7f800000);
  for (unsigned c = 0; c < p.n_splits; ++c)
    M = fmaxf(M, p.part_m[(kvh * p.n_splits + c) * kGroup + hl]);
  float L = 0.0f, o = 0.0f;
  for (unsigned c = 0; c < p.n_splits; ++c) {
    const size_t i = (size_t(kvh) * p.n_splits + c) * kGroup + hl;
    const float w = __expf(p.part_m[i] - M);
    L += w * p.part_l[i];
    o += w * p.part_o[i * kDim + d];
  }
  const unsigned tile = h * (kDim / 64) + d / 64;
  if (tile >= first_tile && tile < first_tile + n_tiles)
    p.core[h * kDim + d] = o / L / (1.0f + __expf(-p.qg[h * 2 * kDim + kDim + d]));
}

template <bool kPrepared, int kPipeline>
__global__ void combine_range(k::AttnCombineParams p, unsigned first, unsigned count) {
  k::attn_combine_op<64, kPrepared, kPipeline>(p, first, count);
}

}  // namespace

extern "C" {

// variant: 0 = <64>, 1 = <64, true>, 4 = <64, true, 4>, 256 = <256>, -1 = serial reference.
// partial != 0: items [5, 52) only, on a 13-block grid (grid-stride tail), for variants 0/1/4.
int test_combine(int variant, int partial, const k::AttnCombineParams* pp, void* stream) {
  const k::AttnCombineParams p = *pp;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned first = partial ? 5 : 0, count = partial ? 47 : 64;
  if (variant == -1) {
    combine_serial<<<16, 256, 0, s>>>(p, first, count);
  } else if (partial) {
    if (variant == 4)
      combine_range<true, 4><<<13, 64, 0, s>>>(p, first, count);
    else if (variant == 1)
      combine_range<true, 1><<<13, 64, 0, s>>>(p, first, count);
    else
      combine_range<false, 1><<<13, 64, 0, s>>>(p, first, count);
  } else if (variant == 4) {
    k::attn_combine_kernel<64, true, 4><<<64, 64, 0, s>>>(p);
  } else if (variant == 1) {
    k::attn_combine_kernel<64, true><<<64, 64, 0, s>>>(p);
  } else if (variant == 256) {
    k::attn_combine_kernel<256><<<16, 256, 0, s>>>(p);
  } else {
    k::attn_combine_kernel<64><<<64, 64, 0, s>>>(p);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
