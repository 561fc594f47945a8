#pragma once

// Batched decode prep: the per-head RMSNorm + partial NEOX RoPE + KV append of attn_prep_kernel
// (kernels/attention_decode.hpp) for a batch of sequences, each at its own position. One block
// per sequence, one warp per head (18 warps), so the block alone owns lens[b] and advances it
// after the append without a race.

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

constexpr int kThreads = 18 * 32;  // one warp per head: 16 query heads, 2 KV heads

__global__ void __launch_bounds__(kThreads) prep_batched_kernel(Args a) {
  using namespace miso::kernels;
  using namespace miso::kernels::attn;
  const unsigned b = blockIdx.x, head = threadIdx.x / 32;
  if (b >= a.batch)
    return;
  const unsigned pos = static_cast<unsigned>(a.lens[b]);
  const float* qg = a.qg + size_t(b) * a.proj_stride;
  const float* kk = a.k + size_t(b) * a.proj_stride;
  const float* vv = a.v + size_t(b) * a.proj_stride;
  if (head < kQHeads) {
    attn_detail::prep_row_warp(qg + head * 2 * kDim, a.q_norm, a.inv_freq, pos, a.eps,
                               a.q + (size_t(b) * kQHeads + head) * kDim, nullptr, nullptr,
                               nullptr);
  } else {
    const unsigned kvh = head - kQHeads;
    const size_t row = size_t(a.kv_row[2 * b + kvh] + pos) * kDim;
    attn_detail::prep_row_warp(kk + kvh * kDim, a.k_norm, a.inv_freq, pos, a.eps, nullptr,
                               a.k_pool + row, vv + kvh * kDim, a.v_pool + row);
  }
  __syncthreads();  // every warp has read lens[b]
  if (threadIdx.x == 0)
    a.lens[b] = static_cast<int32_t>(pos + 1);
}

// Prefill prep for the tensor-core prefill: attn_prep_batch_kernel (kernels/attention_prefill.hpp)
// with the queries stored as fp16 [n][16][256] (the operand type of the tcgen05 prefill). One block
// per kPrepTokens tokens, one warp per head; each warp issues the loads of all its tokens before
// the first row's arithmetic. The rotation angles depend only on the position, so warp i < 4
// computes token i's 32 (sin, cos) pairs once (one per lane) for all 18 heads: the drop-in prep
// spends most of its instructions on 8 serial sincosf in 8 lanes of every row. Same arithmetic as
// the drop-in prep (attn_detail::prep_row_math) up to the final rounding.
struct PrefillArgs {
  const float* qg;
  const float* k;
  const float* v;
  const float* q_norm;
  const float* k_norm;
  const float* inv_freq;
  __half* k_cache;
  __half* v_cache;
  __half* q16;
  unsigned pos0, max_ctx, n, proj_stride;
  float eps;
};

constexpr unsigned kPrepTokens = 4;

__global__ void __launch_bounds__(kThreads) prefill_prep_kernel(PrefillArgs a) {
  using namespace miso::kernels;
  using namespace miso::kernels::attn;
  const unsigned t0 = blockIdx.x * kPrepTokens, head = threadIdx.x / 32;
  if (t0 >= a.n)
    return;
  const unsigned nt = min(kPrepTokens, a.n - t0);
  const bool is_q = head < kQHeads;
  const unsigned kvh = head - kQHeads;
  const float* src0 = is_q ? a.qg + head * 2 * kDim : a.k + kvh * kDim;
  __shared__ float2 sc[kPrepTokens][kRopeDim / 2];
  if (head < kPrepTokens && head < nt) {
    const unsigned lane = threadIdx.x % 32;
    float sn, cs;
    sincosf(static_cast<float>(a.pos0 + t0 + head) * a.inv_freq[lane], &sn, &cs);
    sc[head][lane] = make_float2(sn, cs);
  }
  float y[kPrepTokens][8], v[kPrepTokens][8], w[8];
  attn_detail::load_row8(is_q ? a.q_norm : a.k_norm, w);
#pragma unroll
  for (unsigned i = 0; i < kPrepTokens; ++i) {
    if (i < nt) {
      const size_t row = size_t(t0 + i) * a.proj_stride;
      attn_detail::load_row8(src0 + row, y[i]);
      if (!is_q)
        attn_detail::load_row8(a.v + row + kvh * kDim, v[i]);
    }
  }
  __syncthreads();  // the (sin, cos) tables
#pragma unroll
  for (unsigned i = 0; i < kPrepTokens; ++i) {
    if (i < nt) {
      const unsigned pos = a.pos0 + t0 + i;
      attn_detail::prep_row_math_table(y[i], w, sc[i], a.eps);
      if (is_q) {
        attn_detail::store_row8_f16(y[i], a.q16 + (size_t(t0 + i) * kQHeads + head) * kDim);
      } else {
        const size_t at = (size_t(kvh) * a.max_ctx + pos) * kDim;
        attn_detail::store_row8_f16(y[i], a.k_cache + at);
        attn_detail::store_row8_f16(v[i], a.v_cache + at);
      }
    }
  }
}

}  // namespace miso::fast::prep
