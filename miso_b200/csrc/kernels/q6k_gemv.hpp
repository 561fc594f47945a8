#pragma once

// Decode GEMV y = W x for Q6_K r1 rows with FP16 activations, the drop-in for the reference's
// kernels/q6k_gemv.hpp (interface :20-25 and :126-129; launched by src/engine/weights.hip:268-279
// as q6k_gemv_kernel<2048, 256, R><<<grid, 256>>>). Same scheme as q4k_gemv.hpp: activations
// staged once per block, one warp per row, 16-byte loads of ql and qh per 32 weights.

#include <cstdint>

#include "gemv_common.hpp"

namespace miso::kernels {

struct Q6kGemvParams {
  const std::uint8_t* w;  // n_rows Q6_K r1 rows of K / 256 blocks
  const float* x;         // K activations
  float* y;               // n_rows outputs
  unsigned n_rows;
};

// Rows [first, first + count); the activations must already be staged in `s`.
template <unsigned K, int kBlock, int kRows = 1>
__device__ inline void q6k_gemv_rows(const Q6kGemvParams& p, unsigned first, unsigned count,
                                     const gemv::StagedX<K>& s, unsigned warp_id,
                                     unsigned warp_count) {
  static_assert(K % 256 == 0 && kBlock % kWave == 0);
  gemv::rows_dot<gemv::Fmt::Q6K, K, kRows>(p.w, p.y, first, count, s, warp_id, warp_count);
}

template <unsigned K, int kBlock, int kRows = 1>
__device__ inline void q6k_gemv_op(const Q6kGemvParams& p, unsigned first, unsigned count) {
  constexpr unsigned kWarps = kBlock / kWave;
  __shared__ gemv::StagedX<K> s;
  gemv::stage_x<gemv::Fmt::Q6K, K, kBlock>(p.x, s);
  q6k_gemv_rows<K, kBlock, kRows>(p, first, count, s, blockIdx.x * kWarps + threadIdx.x / kWave,
                                  gridDim.x * kWarps);
}

template <unsigned K, int kBlock, int kRows = 1>
__global__ void __launch_bounds__(kBlock) q6k_gemv_kernel(Q6kGemvParams p) {
  q6k_gemv_op<K, kBlock, kRows>(p, 0, p.n_rows);
}

}  // namespace miso::kernels
