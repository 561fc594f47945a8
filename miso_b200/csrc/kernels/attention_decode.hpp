#pragma once

// Drop-in CUDA (sm_100a) counterpart of the reference header kernels/attention_decode.hpp:
// gated full attention (qwen3_5_moe), decode path — 16 query heads, 2 KV heads, head_dim 256,
// partial NEOX RoPE on the first 64 dims, fp16 KV cache.
//
// Names, Params layouts and launch conventions are the reference's (kernels/attention_decode.hpp
// :14-309), so src/engine/attention.hip and tests/test_attn_splitk.hip compile unchanged:
// caller-chosen grid, block = kBlock, no dynamic shared memory, grid-stride over work items.
// The bodies are written for 32-lane CUDA warps. The B200 fast path (TMA-fed, tensor-core,
// stream-K batched decode) sits behind miso_attn_decode() in include/miso_cuda.h; these templates
// are the portable implementation for callers that launch the reference names themselves.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "wave.hpp"

namespace miso::kernels {

namespace attn {
constexpr int kQHeads = 16, kKvHeads = 2, kDim = 256, kRopeDim = 64;
// The reference uses _Float16; nvcc device code needs __half (same 2-byte IEEE binary16 layout,
// and static_cast<half_t>(float) / static_cast<float>(h) / bit casts work on the host too).
typedef __half half_t;
}  // namespace attn

struct AttnPrepParams {
  const float* qg;        // [16][512]: per head 256 query then 256 gate
  const float* k;         // [2][256]
  const float* v;         // [2][256]
  const float* q_norm;    // [256], stores 1 + w
  const float* k_norm;    // [256]
  const float* inv_freq;  // [32]
  attn::half_t* k_cache;  // [2][max_ctx][256]
  attn::half_t* v_cache;  // [2][max_ctx][256]
  float* q;               // [16][256] normalised, rotated queries
  unsigned pos, max_ctx;
  float eps;
};

// Prefill form: token t reads qg / k / v at `t * proj_stride` floats past tok0's pointers.
struct AttnPrepBatchParams {
  AttnPrepParams tok0;
  unsigned n;
  unsigned proj_stride;
};

namespace attn_detail {

// RMSNorm with `w` and the NEOX rotation of dims [0, 64) at position `pos` of one row of 256 held
// by a warp, lane l owning dims [8l, 8l + 8) in y (dim d < 32 pairs with d + 32, i.e. lane l < 4
// with lane l + 4). Warp-synchronous.
__device__ __forceinline__ void prep_row_math(float (&y)[8], const float (&w)[8],
                                              const float* inv_freq, unsigned pos, float eps) {
  using namespace attn;
  const unsigned lane = threadIdx.x % kWave;
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    ss += y[i] * y[i];
  const float inv_rms = rsqrtf(wave_sum(ss) / kDim + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    y[i] = y[i] * inv_rms * w[i];
  float partner[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    partner[i] = __shfl_xor_sync(0xffffffffu, y[i], 4);
  if (lane < kRopeDim / 8) {
    constexpr unsigned kHalf = kRopeDim / 2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const unsigned d = 8 * lane + i;
      float sn, cs;
      sincosf(static_cast<float>(pos) * inv_freq[d % kHalf], &sn, &cs);
      y[i] = d < kHalf ? y[i] * cs - partner[i] * sn : y[i] * cs + partner[i] * sn;
    }
  }
}

// prep_row_math with the rotation's (sin, cos) taken from a table: sc[f] = sincos(pos *
// inv_freq[f]) for the 32 frequencies f of the position (the same values prep_row_math computes,
// so the results are identical; the table is shared by all heads of a token).
__device__ __forceinline__ void prep_row_math_table(float (&y)[8], const float (&w)[8],
                                                    const float2* sc, float eps) {
  using namespace attn;
  const unsigned lane = threadIdx.x % kWave;
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    ss += y[i] * y[i];
  const float inv_rms = rsqrtf(wave_sum(ss) / kDim + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    y[i] = y[i] * inv_rms * w[i];
  float partner[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    partner[i] = __shfl_xor_sync(0xffffffffu, y[i], 4);
  if (lane < kRopeDim / 8) {
    constexpr unsigned kHalf = kRopeDim / 2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const unsigned d = 8 * lane + i;
      const float2 t = sc[d % kHalf];
      y[i] = d < kHalf ? y[i] * t.y - partner[i] * t.x : y[i] * t.y + partner[i] * t.x;
    }
  }
}

// Lane's 8 consecutive floats of a row of 256.
__device__ __forceinline__ void load_row8(const float* row, float (&y)[8]) {
  const float4* r4 = reinterpret_cast<const float4*>(row) + 2 * (threadIdx.x % kWave);
  const float4 a = r4[0], b = r4[1];
  y[0] = a.x, y[1] = a.y, y[2] = a.z, y[3] = a.w, y[4] = b.x, y[5] = b.y, y[6] = b.z, y[7] = b.w;
}

// Lane's 8 values of a row of 256 as fp16 (one 16-byte store).
__device__ __forceinline__ void store_row8_f16(const float (&y)[8], attn::half_t* row) {
  __align__(16) __half h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    h[i] = __float2half_rn(y[i]);
  reinterpret_cast<uint4*>(row)[threadIdx.x % kWave] = *reinterpret_cast<const uint4*>(h);
}

// One row of 256 (a query head or a key head) on one warp: prep_row_math, then either an fp32
// store (out_f32) or an fp16 store (out_f16, plus the matching value row v_src -> v_dst when
// v_src is given). Warp-synchronous, no shared memory, so the drop-in and batched prep kernels
// produce identical bits.
__device__ __forceinline__ void prep_row_warp(const float* src, const float* weight,
                                              const float* inv_freq, unsigned pos, float eps,
                                              float* out_f32, attn::half_t* out_f16,
                                              const float* v_src, attn::half_t* v_dst) {
  float y[8], w[8];
  load_row8(src, y);
  load_row8(weight, w);
  prep_row_math(y, w, inv_freq, pos, eps);
  if (out_f32 != nullptr) {
    float4* o4 = reinterpret_cast<float4*>(out_f32) + 2 * (threadIdx.x % kWave);
    o4[0] = make_float4(y[0], y[1], y[2], y[3]);
    o4[1] = make_float4(y[4], y[5], y[6], y[7]);
  } else {
    store_row8_f16(y, out_f16);
    if (v_src == nullptr)
      return;
    float v[8];
    load_row8(v_src, v);
    store_row8_f16(v, v_dst);
  }
}

}  // namespace attn_detail

// Head `head` of 18 (0..15 query heads, 16..17 KV heads): norm, RoPE at p.pos, then store q or
// append k / v at cache position p.pos. The first warp of the block does the row.
template <int kBlock>
__device__ void attn_prep_head(const AttnPrepParams& p, unsigned head) {
  using namespace attn;
  static_assert(kBlock % kWave == 0, "whole warps");
  if (threadIdx.x >= kWave)
    return;
  if (head < kQHeads) {
    attn_detail::prep_row_warp(p.qg + head * 2 * kDim, p.q_norm, p.inv_freq, p.pos, p.eps,
                               p.q + head * kDim, nullptr, nullptr, nullptr);
  } else {
    const unsigned kvh = head - kQHeads;
    const std::size_t at = (std::size_t{kvh} * p.max_ctx + p.pos) * kDim;
    attn_detail::prep_row_warp(p.k + kvh * kDim, p.k_norm, p.inv_freq, p.pos, p.eps, nullptr,
                               p.k_cache + at, p.v + kvh * kDim, p.v_cache + at);
  }
}

// Heads [first, first + count) of 18, one block per head, grid-stride.
template <int kBlock>
__device__ void attn_prep_op(const AttnPrepParams& p, unsigned first, unsigned count) {
  for (unsigned head = first + blockIdx.x; head < first + count; head += gridDim.x)
    attn_prep_head<kBlock>(p, head);
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) attn_prep_kernel(AttnPrepParams p) {
  attn_prep_op<kBlock>(p, 0, attn::kQHeads + attn::kKvHeads);
}

// ---- split-K decode ---------------------------------------------------------------------------

constexpr unsigned kAttnSubChunk = 32;

// Split count per KV head (the reference policy, kernels/attention_decode.hpp:95-115, kept
// identical because callers size scratch with it and tests pin its values): aim for six
// 32-position sub-chunks per split; above max_splits, spread the sub-chunks evenly over
// max_splits; below 16 splits (when max_splits allows 16), use one split per sub-chunk up to 16.
__host__ __device__ constexpr unsigned attn_n_splits(unsigned len, unsigned max_splits) {
  const unsigned subs = (len + kAttnSubChunk - 1) / kAttnSubChunk;
  if (subs == 0)
    return 1;
  unsigned per = 6;
  unsigned splits = (subs + per - 1) / per;
  if (splits > max_splits) {
    per = (subs + max_splits - 1) / max_splits;
  } else if (splits < 16 && max_splits >= 16) {
    const unsigned want = subs < 16 ? subs : 16u;
    if (splits < want)
      per = (subs + want - 1) / want;
  }
  return (subs + per - 1) / per;
}

struct AttnSplitParams {
  const float* q;               // [16][256] (unscaled)
  const attn::half_t* k_cache;  // [2][max_ctx][256]
  const attn::half_t* v_cache;
  float* part_m;  // [2][n_splits][8] running max of scaled scores
  float* part_l;  // [2][n_splits][8] sum of exp(score - max)
  float* part_o;  // [2][n_splits][8][256] sum of exp(score - max) V
  unsigned len, max_ctx, n_splits;
};

// Items [first, first + count) with item = kvh * n_splits + split. Split `split` covers the
// positions [split * per * 32, min(len, (split + 1) * per * 32)) with per = ceil(subs / n_splits).
// One warp per query head of the KV group: in the score phase lane j owns key j of a 32-key
// sub-chunk (K staged in padded shared rows, conflict-free); in the value phase lane i owns
// dims [8i, 8i + 8) and the probabilities are broadcast by shuffle. The online softmax state
// (max, sum) is warp-uniform and lives in registers.
template <int kBlock>
__device__ void attn_split_op(const AttnSplitParams& p, unsigned first, unsigned count) {
  using namespace attn;
  constexpr int kGroup = kQHeads / kKvHeads, kSub = kAttnSubChunk;
  constexpr int kKRow = kDim / 2 + 1;  // half2 per padded K row: 129 words
  static_assert(kBlock == kGroup * kWave, "one warp per query head of the KV group");
  static_assert(kSub == kWave, "one lane per key of a sub-chunk");
  __shared__ float qs[kGroup][kDim];
  __shared__ __half2 ks[kSub][kKRow];
  __shared__ __align__(16) uint4 vs[kSub][kDim / 8];
  const unsigned tid = threadIdx.x, lane = tid % kWave, h = tid / kWave;
  const float scale = rsqrtf(static_cast<float>(kDim));
  const unsigned subs = (p.len + kSub - 1) / kSub;
  const unsigned per = (subs + p.n_splits - 1) / p.n_splits;

  for (unsigned item = first + blockIdx.y * gridDim.x + blockIdx.x; item < first + count;
       item += gridDim.x * gridDim.y) {
    const unsigned kvh = item / p.n_splits, split = item % p.n_splits;
    const __half2* K = reinterpret_cast<const __half2*>(p.k_cache + std::size_t{kvh} * p.max_ctx * kDim);
    const uint4* V = reinterpret_cast<const uint4*>(p.v_cache + std::size_t{kvh} * p.max_ctx * kDim);
    for (unsigned i = tid; i < kGroup * kDim; i += kBlock)
      qs[i / kDim][i % kDim] = p.q[kvh * kGroup * kDim + i] * scale;
    float m = -__int_as_float(0x7f800000), l = 0.0f, acc[8] = {};
    const unsigned j_begin = split * per * kSub;
    const unsigned j_end = min(p.len, (split + 1) * per * kSub);
    __syncthreads();

    for (unsigned j0 = j_begin; j0 < j_end; j0 += kSub) {
      const unsigned n = min(static_cast<unsigned>(kSub), j_end - j0);
      for (unsigned e = tid; e < kSub * (kDim / 2); e += kBlock) {
        const unsigned r = e / (kDim / 2), c = e % (kDim / 2);
        if (r < n)
          ks[r][c] = K[std::size_t{j0 + r} * (kDim / 2) + c];
      }
      for (unsigned e = tid; e < kSub * (kDim / 8); e += kBlock) {
        const unsigned r = e / (kDim / 8), c = e % (kDim / 8);
        if (r < n)
          vs[r][c] = V[std::size_t{j0 + r} * (kDim / 8) + c];
      }
      __syncthreads();
      float s = -__int_as_float(0x7f800000);
      if (lane < n) {
        s = 0.0f;
#pragma unroll 8
        for (int e = 0; e < kDim / 2; ++e) {
          const float2 kf = __half22float2(ks[lane][e]);
          s += qs[h][2 * e] * kf.x + qs[h][2 * e + 1] * kf.y;
        }
      }
      const float m_new = fmaxf(m, wave_max(s));
      const float pj = lane < n ? __expf(s - m_new) : 0.0f;
      const float corr = __expf(m - m_new);
      l = l * corr + wave_sum(pj);
      m = m_new;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        acc[c] *= corr;
      for (unsigned j = 0; j < n; ++j) {
        const float pb = __shfl_sync(0xffffffffu, pj, j);
        const uint4 raw = vs[j][lane];
        const __half2* hv = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 vf = __half22float2(hv[c]);
          acc[2 * c] += pb * vf.x;
          acc[2 * c + 1] += pb * vf.y;
        }
      }
      __syncthreads();
    }
    const std::size_t base = (std::size_t{kvh} * p.n_splits + split) * kGroup + h;
    if (lane == 0)
      p.part_m[base] = m, p.part_l[base] = l;
    float4* o4 = reinterpret_cast<float4*>(p.part_o + base * kDim + 8 * lane);
    o4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    __syncthreads();
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) attn_split_kernel(AttnSplitParams p) {
  attn_split_op<kBlock>(p, 0, attn::kKvHeads * p.n_splits);
}

// ---- gated combine ----------------------------------------------------------------------------

struct AttnCombineParams {
  const float* part_m;
  const float* part_l;
  const float* part_o;
  const float* qg;  // [16][512], for the gate half
  float* core;      // [16][256] = softmax(q K^T / 16) V * sigmoid(gate)
  unsigned n_splits;
};

// Items [first, first + count) = (head, tile of kBlock dims). Every variant evaluates exactly
// M = max_c m_c;  w_c = __expf(m_c - M);  L += w_c * l_c;  o += w_c * o_c  (c ascending);
// core = o / L / (1 + __expf(-gate)), so all variants agree bit for bit (the reference's combine
// contract, tests/test_attn_splitk.hip:22-40,180-187). kPrepared: with n_splits <= 32 each lane of
// a warp computes one split's weight once and the ordered sum takes it by shuffle; kPipeline = 4
// issues four part_o loads ahead of their use.
template <int kBlock, bool kPrepared = false, int kPipeline = 1>
__device__ void attn_combine_op(const AttnCombineParams& p, unsigned first, unsigned count) {
  using namespace attn;
  constexpr int kGroup = kQHeads / kKvHeads, kTiles = kDim / kBlock;
  static_assert(kDim % kBlock == 0 && kBlock % kWave == 0, "whole warps tiling 256 dims");
  static_assert(kPipeline == 1 || (kPrepared && kPipeline == 4), "pipeline needs prepared");
  const unsigned lane = threadIdx.x % kWave;
  for (unsigned item = first + blockIdx.x; item < first + count; item += gridDim.x) {
    const unsigned h = item / kTiles, d = (item % kTiles) * kBlock + threadIdx.x;
    const unsigned kvh = h / kGroup, hl = h % kGroup;
    const std::size_t head0 = std::size_t{kvh} * p.n_splits * kGroup + hl;  // split c at + c * 8
    float L = 0.0f, o = 0.0f;
    if (kPrepared && p.n_splits <= static_cast<unsigned>(kWave)) {
      const bool live = lane < p.n_splits;
      const float m_lane = live ? p.part_m[head0 + lane * kGroup] : -__int_as_float(0x7f800000);
      const float M = wave_max(m_lane);
      const float w_lane = live ? __expf(m_lane - M) : 0.0f;
      const float l_lane = live ? p.part_l[head0 + lane * kGroup] : 0.0f;
      unsigned c = 0;
      for (; c + kPipeline <= p.n_splits; c += kPipeline) {
        float x[kPipeline];
#pragma unroll
        for (int r = 0; r < kPipeline; ++r)
          x[r] = p.part_o[(head0 + (c + r) * kGroup) * kDim + d];
#pragma unroll
        for (int r = 0; r < kPipeline; ++r) {
          const float w = __shfl_sync(0xffffffffu, w_lane, c + r);
          const float lc = __shfl_sync(0xffffffffu, l_lane, c + r);
          L += w * lc;
          o += w * x[r];
        }
      }
      for (; c < p.n_splits; ++c) {
        const float w = __shfl_sync(0xffffffffu, w_lane, c);
        const float lc = __shfl_sync(0xffffffffu, l_lane, c);
        L += w * lc;
        o += w * p.part_o[(head0 + c * kGroup) * kDim + d];
      }
    } else {
      float M = -__int_as_float(0x7f800000);
      for (unsigned c = 0; c < p.n_splits; ++c)
        M = fmaxf(M, p.part_m[head0 + c * kGroup]);
      for (unsigned c = 0; c < p.n_splits; ++c) {
        const std::size_t i = head0 + c * kGroup;
        const float w = __expf(p.part_m[i] - M);
        L += w * p.part_l[i];
        o += w * p.part_o[i * kDim + d];
      }
    }
    const float gate = p.qg[h * 2 * kDim + kDim + d];
    p.core[h * kDim + d] = o / L / (1.0f + __expf(-gate));
  }
}

template <int kBlock, bool kPrepared = false, int kPipeline = 1>
__global__ void __launch_bounds__(kBlock) attn_combine_kernel(AttnCombineParams p) {
  attn_combine_op<kBlock, kPrepared, kPipeline>(p, 0, attn::kQHeads * (attn::kDim / kBlock));
}

}  // namespace miso::kernels
