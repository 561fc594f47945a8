#pragma once

// Two independent decode projections of one activation vector in one launch: a Q6_K r1 matrix and
// a Q4_K r1 matrix, both K = 2048 — the drop-in for the reference's kernels/mixed_gemv.hpp
// (interface :12-28; launched by src/engine/weights.hip:293-299 as
// mixed_gemv_kernel<R6, G6, G4><<<G6 + G4, 256>>>(p6, p4)). Blocks [0, Q6Grid) run the Q6_K GEMV
// as if it had a grid of Q6Grid blocks (Q6Rows rows per warp step), blocks [Q6Grid, Q6Grid +
// Q4Grid) the Q4_K GEMV with a grid of Q4Grid (4 rows per warp step). Each block stages the
// activations in the chunk order of the format it computes.

#include "q4k_gemv.hpp"
#include "q6k_gemv.hpp"

namespace miso::kernels {

template <int Q6Rows, unsigned Q6Grid, unsigned Q4Grid, int kBlock = 256>
__device__ inline void mixed_gemv_op(const Q6kGemvParams& q6, const Q4kGemvParams& q4) {
  constexpr unsigned K = 2048, kWarps = kBlock / kWave;
  __shared__ gemv::StagedX<K> s;
  const unsigned warp = threadIdx.x / kWave;
  if (blockIdx.x < Q6Grid) {  // uniform over the block
    gemv::stage_x<gemv::Fmt::Q6K, K, kBlock>(q6.x, s);
    gemv::rows_dot<gemv::Fmt::Q6K, K, Q6Rows>(q6.w, q6.y, 0, q6.n_rows, s,
                                               blockIdx.x * kWarps + warp, Q6Grid * kWarps);
  } else {
    gemv::stage_x<gemv::Fmt::Q4K, K, kBlock>(q4.x, s);
    gemv::rows_dot<gemv::Fmt::Q4K, K, 4>(q4.w, q4.y, 0, q4.n_rows, s,
                                          (blockIdx.x - Q6Grid) * kWarps + warp, Q4Grid * kWarps);
  }
}

template <int Q6Rows, unsigned Q6Grid, unsigned Q4Grid, int kBlock = 256>
__global__ void __launch_bounds__(kBlock) mixed_gemv_kernel(Q6kGemvParams q6, Q4kGemvParams q4) {
  mixed_gemv_op<Q6Rows, Q6Grid, Q4Grid, kBlock>(q6, q4);
}

}  // namespace miso::kernels
