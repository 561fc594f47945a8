#pragma once

// Decode GEMV y = W x for Q4_K r1 weights, the drop-in for the reference's kernels/q4k_gemv.hpp
// (interface :18-28 and :234-237; launched by src/engine/weights.hip:256-267 as
// q4k_gemv_kernel<ActFormat::Fp16, K, 256, R><<<grid, 256>>>).
//
// Each block stages the K activations once in shared memory (converted to the activation format,
// in the chunk order of gemv_common.hpp), then its warps stride over groups of kRows rows of the
// grid: one warp per row, each lane one 16-byte load of nibbles (32 weights) per 1024 weights of
// the row, with every load of the group's rows issued before the arithmetic.

#include <cstdint>

#include "gemv_common.hpp"

namespace miso::kernels {

enum class ActFormat {
  Int8,  // per-32 absmax INT8 activations
  Fp16,  // FP16 activations
};

struct Q4kGemvParams {
  const std::uint8_t* w;  // n_rows rows of K / 256 Q4_K r1 blocks (144 bytes each)
  const float* x;         // K activations
  float* y;               // n_rows outputs
  unsigned n_rows;
};

namespace gemv {
template <ActFormat A>
inline constexpr Act act_of = A == ActFormat::Int8 ? Act::Int8 : Act::Fp16;
}  // namespace gemv

// Rows [first, first + count); the activations must already be staged in `s`.
template <unsigned K, int kBlock, int kRows = 1>
__device__ inline void q4k_gemv_rows(const Q4kGemvParams& p, unsigned first, unsigned count,
                                     const gemv::StagedX<K>& s, unsigned warp_id,
                                     unsigned warp_count) {
  static_assert(K % 256 == 0 && kBlock % kWave == 0);
  gemv::rows_dot<gemv::Fmt::Q4K, K, kRows>(p.w, p.y, first, count, s, warp_id, warp_count);
}

// Rows [first, first + count): stages x, then computes.
template <ActFormat A, unsigned K, int kBlock, int kRows = 1>
__device__ inline void q4k_gemv_op(const Q4kGemvParams& p, unsigned first, unsigned count) {
  constexpr unsigned kWarps = kBlock / kWave;
  __shared__ gemv::StagedX<K> s;
  gemv::stage_x<gemv::Fmt::Q4K, K, kBlock, gemv::act_of<A>>(p.x, s);
  q4k_gemv_rows<K, kBlock, kRows>(p, first, count, s, blockIdx.x * kWarps + threadIdx.x / kWave,
                                  gridDim.x * kWarps);
}

template <ActFormat A, unsigned K, int kBlock, int kRows = 1>
__global__ void __launch_bounds__(kBlock) q4k_gemv_kernel(Q4kGemvParams p) {
  q4k_gemv_op<A, K, kBlock, kRows>(p, 0, p.n_rows);
}

}  // namespace miso::kernels
