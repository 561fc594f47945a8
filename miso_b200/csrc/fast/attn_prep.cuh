#pragma once

// Batched decode prep: the per-head RMSNorm + partial NEOX RoPE + KV append of attn_prep_kernel
// (kernels/attention_decode.hpp) for a batch of sequences, each at its own position. One block
// per sequence, one warp per head (18 warps), so the block alone owns lens[b] and advances it
// after the append without a race (every warp has read lens[b] at the block barrier).

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
  const unsigned b = blockIdx.x, head = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (b >= a.batch)
    return;
  const unsigned pos = static_cast<unsigned>(a.lens[b]);
  const float* qg = a.qg + size_t(b) * a.proj_stride;
  const float* kk = a.k + size_t(b) * a.proj_stride;
  const float* vv = a.v + size_t(b) * a.proj_stride;
  const bool is_q = head < kQHeads;
  const unsigned kvh = head - kQHeads;
  float y[8], w[8];
  attn_detail::load_row8(is_q ? qg + head * 2 * kDim : kk + kvh * kDim, y);
  attn_detail::load_row8(is_q ? a.q_norm : a.k_norm, w);
  // The rotation's (sin, cos) depend only on the position: computed once (one per lane) for all
  // 18 heads, with the same sincosf arguments as attn_detail::prep_row_math.
  __shared__ float2 sc[kRopeDim / 2];
  if (head == 0) {
    float sn, cs;
    sincosf(static_cast<float>(pos) * a.inv_freq[lane], &sn, &cs);
    sc[lane] = make_float2(sn, cs);
  }
  __syncthreads();  // the table; also: every warp has read lens[b]
  attn_detail::prep_row_math_table(y, w, sc, a.eps);
  if (is_q) {
    float4* o4 = reinterpret_cast<float4*>(a.q + (size_t(b) * kQHeads + head) * kDim) + 2 * lane;
    o4[0] = make_float4(y[0], y[1], y[2], y[3]);
    o4[1] = make_float4(y[4], y[5], y[6], y[7]);
  } else {
    const size_t row = size_t(a.kv_row[2 * b + kvh] + pos) * kDim;
    attn_detail::store_row8_f16(y, a.k_pool + row);
    float v[8];
    attn_detail::load_row8(vv + kvh * kDim, v);
    attn_detail::store_row8_f16(v, a.v_pool + row);
  }
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
