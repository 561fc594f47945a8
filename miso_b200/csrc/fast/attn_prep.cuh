#pragma once

// Batched decode prep: the per-head RMSNorm + partial NEOX RoPE + KV append of attn_prep_kernel
// (kernels/attention_decode.hpp) for a batch of sequences, each at its own position. One
// 256-thread block per sequence walks its 18 heads, so the block alone owns lens[b] and can
// advance it after the append without a race.

#include <cuda_runtime.h>

#include <cstdint>

#include "../kernels/attention_decode.hpp"

namespace miso::fast::prep {

struct Args {
  const float* qg;
  const float* k;
  const float* v;
  const float* q_norm;
  const float* k_norm;
  const float* inv_freq;
  __half* k_pool;
  __half* v_pool;
  const int64_t* kv_row;
  int32_t* lens;
  float* q;
  unsigned batch;
  unsigned proj_stride;
  float eps;
};

__global__ void __launch_bounds__(256) prep_batched_kernel(Args a) {
  using namespace miso::kernels;
  using namespace miso::kernels::attn;
  const unsigned b = blockIdx.x;
  if (b >= a.batch)
    return;
  const unsigned pos = static_cast<unsigned>(a.lens[b]);
  const float* qg = a.qg + size_t(b) * a.proj_stride;
  const float* kk = a.k + size_t(b) * a.proj_stride;
  const float* vv = a.v + size_t(b) * a.proj_stride;
  for (unsigned head = 0; head < kQHeads + kKvHeads; ++head) {
    if (head < kQHeads) {
      attn_detail::prep_row<256>(qg + head * 2 * kDim, a.q_norm, a.inv_freq, pos, a.eps,
                                 a.q + (size_t(b) * kQHeads + head) * kDim, nullptr, nullptr,
                                 nullptr);
    } else {
      const unsigned kvh = head - kQHeads;
      const size_t row = size_t(a.kv_row[2 * b + kvh] + pos) * kDim;
      attn_detail::prep_row<256>(kk + kvh * kDim, a.k_norm, a.inv_freq, pos, a.eps, nullptr,
                                 a.k_pool + row, vv + kvh * kDim, a.v_pool + row);
    }
  }
  // prep_row ends with a barrier, so every thread has read lens[b] already.
  if (threadIdx.x == 0)
    a.lens[b] = static_cast<int32_t>(pos + 1);
}

}  // namespace miso::fast::prep
