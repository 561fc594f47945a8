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

#include "../common/warp_mma.cuh"
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

namespace attn_detail {

// Merge slot of the split kernel: [8 heads][256 dims] fp32 then l[8]. Dims are stored in rows of
// 33 per group of 32 and heads 268 floats apart, so the stores of a fragment (lane (g, tq):
// heads 2 tq, 2 tq + 1, dims 32 g + ...) fall in 32 different banks.
constexpr int kSplitSlotHead = 268;
constexpr int kSplitSlotFloats = 8 * kSplitSlotHead + 8;
__device__ __forceinline__ int split_slot_index(unsigned h, unsigned d) {
  return int(h) * kSplitSlotHead + int(d / 32) * 33 + int(d % 32);
}

}  // namespace attn_detail

// Items [first, first + count) with item = kvh * n_splits + split. Split `split` covers the
// positions [split * per * 32, min(len, (split + 1) * per * 32)) with per = ceil(subs / n_splits)
// (the reference partition; the combine merges the splits' (max, sum, output) triples).
//
// Tensor-core body inside the caller's geometry (kBlock = 256 threads = 8 warps, no dynamic shared
// memory). The split's keys are cut into 16-key slabs; warp w takes slabs w, w + 8, ... and
// streams each slab straight from global memory into mma.sync m16n8k16 fragments (no shared-
// memory staging, so each warp has a whole slab of K and V - 16 KB - in flight, and the next
// slab's loads are issued while the current one is computed):
//   S^T[16 keys][8 heads] = K Q^T      with the head dimension permuted so that a lane's K
//                                      fragment elements are its 64 contiguous dims
//                                      [64 tq, 64 tq + 64) of keys g and g + 8 (eight 16-byte
//                                      loads per key); Q uses the same permutation
//   O^T[256 dims][8 heads] += V^T P^T  with the output dims permuted so that a lane reads dims
//                                      [32 g, 32 g + 32) of keys 2 tq, 2 tq + 1, 2 tq + 8,
//                                      2 tq + 9, and pairs the two keys' halves by byte permutes
// (g = lane / 4, tq = lane % 4). The fp32 query and the probabilities are split into fp16 high and
// low parts (two MMAs each; K and V are exact fp16), so the result keeps fp32 accuracy; the online
// softmax is per warp, and the eight warp states are merged through shared memory at the end.
template <int kBlock>
__device__ void attn_split_op(const AttnSplitParams& p, unsigned first, unsigned count) {
  using namespace attn;
  using attn_detail::kSplitSlotFloats;
  using attn_detail::split_slot_index;
  constexpr int kGroup = kQHeads / kKvHeads, kSlab = 16, kWarps = kBlock / kWave;
  static_assert(kBlock == kGroup * kWave && kWave == 32, "eight 32-lane warps");
  __shared__ uint4 qfrag[16][32];  // per k-step and lane: Q^T fragments {hi b0, hi b1, lo b0, lo b1}
  __shared__ float slot[2][kSplitSlotFloats];
  __shared__ float red_m[kWarps][kGroup];
  const unsigned tid = threadIdx.x, warp = tid / kWave, lane = tid % kWave;
  const unsigned g = lane / 4, tq = lane % 4;
  const float kNegInf = -__int_as_float(0x7f800000);
  const unsigned subs = (p.len + kAttnSubChunk - 1) / kAttnSubChunk;
  const unsigned per = (subs + p.n_splits - 1) / p.n_splits;
  const uint64_t policy = dev::stream_policy();

  for (unsigned item = first + blockIdx.y * gridDim.x + blockIdx.x; item < first + count;
       item += gridDim.x * gridDim.y) {
    const unsigned kvh = item / p.n_splits, split = item % p.n_splits;
    const half_t* K = p.k_cache + std::size_t{kvh} * p.max_ctx * kDim;
    const half_t* V = p.v_cache + std::size_t{kvh} * p.max_ctx * kDim;
    const unsigned j_begin = split * per * kAttnSubChunk;
    const unsigned j_end = min(p.len, (split + 1) * per * kAttnSubChunk);
    const unsigned nslab = j_end > j_begin ? (j_end - j_begin + kSlab - 1) / kSlab : 0;

    // Q^T fragments of the group's 8 heads (pre-scaled by 1/16, exact): k-step ks, lane (fg, ft)
    // holds dims 64 ft + 4 ks + {0, 1} (b0) and + {2, 3} (b1) of head fg, as fp16 hi and lo.
    for (unsigned e = tid; e < 16 * 32; e += kBlock) {
      const unsigned ks = e / 32, ln = e % 32, fg = ln / 4, ft = ln % 4;
      const float4 x = *reinterpret_cast<const float4*>(p.q + (kvh * kGroup + fg) * kDim +
                                                        64 * ft + 4 * ks);
      uint4 f;
      dev::split_half2(x.x * 0.0625f, x.y * 0.0625f, f.x, f.z);
      dev::split_half2(x.z * 0.0625f, x.w * 0.0625f, f.y, f.w);
      qfrag[ks][ln] = f;
    }
    __syncthreads();

    float o[16][4];
#pragma unroll
    for (int mb = 0; mb < 16; ++mb)
      o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.0f;
    float m0 = kNegInf, m1 = kNegInf, l0 = 0.0f, l1 = 0.0f;

    // K rows g, g + 8 of a slab: dims [64 tq, +64) as 8 x 16 bytes each; V rows 2 tq, 2 tq + 1,
    // 2 tq + 8, 2 tq + 9: dims [32 g, +32) as 4 x 16 bytes each. Rows at or past j_end are not
    // read (zero).
    uint4 kr[2][8], vr[4][4];
    auto load_k = [&](unsigned s) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const unsigned key = j_begin + kSlab * s + g + 8 * r;
        const half_t* row = K + std::size_t{key} * kDim + 64 * tq;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          kr[r][c] = key < j_end ? dev::ld_stream16(row + 8 * c, policy) : make_uint4(0, 0, 0, 0);
      }
    };
    auto load_v = [&](unsigned s) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const unsigned key = j_begin + kSlab * s + 2 * tq + (r & 1) + 8 * (r >> 1);
        const half_t* row = V + std::size_t{key} * kDim + 32 * g;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          vr[r][c] = key < j_end ? dev::ld_stream16(row + 8 * c, policy) : make_uint4(0, 0, 0, 0);
      }
    };
    auto word = [](const uint4& v, int i) -> uint32_t {
      return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
    };

    if (warp < nslab) {
      load_k(warp);
      load_v(warp);
    }
    for (unsigned s = warp; s < nslab; s += kWarps) {
      const unsigned key0 = j_begin + kSlab * s;
      // ---- S^T = K Q^T (hi and lo query parts in separate accumulators) ----------------------
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 16; ++ks) {
        const uint32_t a0 = word(kr[0][ks / 2], 2 * (ks % 2));
        const uint32_t a2 = word(kr[0][ks / 2], 2 * (ks % 2) + 1);
        const uint32_t a1 = word(kr[1][ks / 2], 2 * (ks % 2));
        const uint32_t a3 = word(kr[1][ks / 2], 2 * (ks % 2) + 1);
        const uint4 qf = qfrag[ks][lane];
        dev::mma_f16(sa, a0, a1, a2, a3, qf.x, qf.y);
        dev::mma_f16(sb, a0, a1, a2, a3, qf.z, qf.w);
      }
      if (s + kWarps < nslab)
        load_k(s + kWarps);  // the K registers are free: start the next slab's keys
      float sv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
        sv[r] = sa[r] + sb[r];
      // sv[0], sv[1]: key g, heads 2 tq, 2 tq + 1; sv[2], sv[3]: key g + 8.
      if (key0 + g >= j_end)
        sv[0] = sv[1] = kNegInf;
      if (key0 + g + 8 >= j_end)
        sv[2] = sv[3] = kNegInf;
      float mx0 = fmaxf(sv[0], sv[2]), mx1 = fmaxf(sv[1], sv[3]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: key0 < j_end
      const float c0 = __expf(m0 - mn0), c1 = __expf(m1 - mn1);
      const float p0 = sv[0] == kNegInf ? 0.0f : __expf(sv[0] - mn0);
      const float p1 = sv[1] == kNegInf ? 0.0f : __expf(sv[1] - mn1);
      const float p2 = sv[2] == kNegInf ? 0.0f : __expf(sv[2] - mn0);
      const float p3 = sv[3] == kNegInf ? 0.0f : __expf(sv[3] - mn1);
      l0 = l0 * c0 + (p0 + p2);
      l1 = l1 * c1 + (p1 + p3);
      m0 = mn0, m1 = mn1;
#pragma unroll
      for (int mb = 0; mb < 16; ++mb)
        o[mb][0] *= c0, o[mb][1] *= c1, o[mb][2] *= c0, o[mb][3] *= c1;
      uint32_t h01, lo01, h23, lo23;
      dev::split_half2(p0, p1, h01, lo01);
      dev::split_half2(p2, p3, h23, lo23);
      const uint32_t bh0 = dev::movmatrix_t(h01), bh1 = dev::movmatrix_t(h23);
      const uint32_t bl0 = dev::movmatrix_t(lo01), bl1 = dev::movmatrix_t(lo23);
      // ---- O^T += V^T P^T: m-block mb, row g = dim 32 g + 2 mb, row g + 8 = the next dim -------
#pragma unroll
      for (int mb = 0; mb < 16; ++mb) {
        const uint32_t w0 = word(vr[0][mb / 4], mb % 4), w1 = word(vr[1][mb / 4], mb % 4);
        const uint32_t w2 = word(vr[2][mb / 4], mb % 4), w3 = word(vr[3][mb / 4], mb % 4);
        const uint32_t a0 = dev::prmt(w0, w1, 0x5410), a1 = dev::prmt(w0, w1, 0x7632);
        const uint32_t a2 = dev::prmt(w2, w3, 0x5410), a3 = dev::prmt(w2, w3, 0x7632);
        dev::mma_f16(o[mb], a0, a1, a2, a3, bh0, bh1);
        dev::mma_f16(o[mb], a0, a1, a2, a3, bl0, bl1);
      }
      if (s + kWarps < nslab)
        load_v(s + kWarps);
    }

    // ---- merge the eight warp states (tree through two shared-memory slots) -------------------
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (g == 0)
      red_m[warp][2 * tq] = m0, red_m[warp][2 * tq + 1] = m1;
    __syncthreads();
    float M0 = kNegInf, M1 = kNegInf;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      M0 = fmaxf(M0, red_m[w][2 * tq]);
      M1 = fmaxf(M1, red_m[w][2 * tq + 1]);
    }
    const float sc0 = m0 == kNegInf ? 0.0f : __expf(m0 - M0);
    const float sc1 = m1 == kNegInf ? 0.0f : __expf(m1 - M1);
    l0 *= sc0, l1 *= sc1;
#pragma unroll
    for (int mb = 0; mb < 16; ++mb)
      o[mb][0] *= sc0, o[mb][1] *= sc1, o[mb][2] *= sc0, o[mb][3] *= sc1;
    auto put = [&](int si) {
      float* sl = slot[si];
#pragma unroll
      for (int mb = 0; mb < 16; ++mb) {
        const unsigned d = 32 * g + 2 * mb;
        sl[split_slot_index(2 * tq, d)] = o[mb][0];
        sl[split_slot_index(2 * tq + 1, d)] = o[mb][1];
        sl[split_slot_index(2 * tq, d + 1)] = o[mb][2];
        sl[split_slot_index(2 * tq + 1, d + 1)] = o[mb][3];
      }
      if (g == 0)
        sl[8 * attn_detail::kSplitSlotHead + 2 * tq] = l0,
        sl[8 * attn_detail::kSplitSlotHead + 2 * tq + 1] = l1;
    };
    auto take = [&](int si) {
      const float* sl = slot[si];
#pragma unroll
      for (int mb = 0; mb < 16; ++mb) {
        const unsigned d = 32 * g + 2 * mb;
        o[mb][0] += sl[split_slot_index(2 * tq, d)];
        o[mb][1] += sl[split_slot_index(2 * tq + 1, d)];
        o[mb][2] += sl[split_slot_index(2 * tq, d + 1)];
        o[mb][3] += sl[split_slot_index(2 * tq + 1, d + 1)];
      }
      l0 += sl[8 * attn_detail::kSplitSlotHead + 2 * tq];
      l1 += sl[8 * attn_detail::kSplitSlotHead + 2 * tq + 1];
    };
    // (w0 + w4) (w1 + w5), (w2 + w6) (w3 + w7), (w0 + w2) (w1 + w3); then slots hold w0, w1.
    if (warp == 4 || warp == 5) put(warp - 4);
    __syncthreads();
    if (warp == 0 || warp == 1) take(warp);
    __syncthreads();
    if (warp == 6 || warp == 7) put(warp - 6);
    __syncthreads();
    if (warp == 2 || warp == 3) take(warp - 2);
    __syncthreads();
    if (warp == 2 || warp == 3) put(warp - 2);
    __syncthreads();
    if (warp == 0 || warp == 1) take(warp);
    __syncthreads();
    if (warp == 0 || warp == 1) put(warp);
    __syncthreads();
    // Write the split's triple: thread (h = tid / 32, dims 8 (tid % 32) .. + 7).
    {
      const unsigned h = tid / 32, d0 = 8 * (tid % 32);
      const std::size_t base = (std::size_t{kvh} * p.n_splits + split) * kGroup + h;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        v[e] = slot[0][split_slot_index(h, d0 + e)] + slot[1][split_slot_index(h, d0 + e)];
      float4* o4 = reinterpret_cast<float4*>(p.part_o + base * kDim + d0);
      o4[0] = make_float4(v[0], v[1], v[2], v[3]);
      o4[1] = make_float4(v[4], v[5], v[6], v[7]);
      if (tid % 32 == 0) {
        float M = kNegInf;
#pragma unroll
        for (int w = 0; w < kWarps; ++w)
          M = fmaxf(M, red_m[w][h]);
        p.part_m[base] = M;
        p.part_l[base] = slot[0][8 * attn_detail::kSplitSlotHead + h] +
                         slot[1][8 * attn_detail::kSplitSlotHead + h];
      }
    }
    __syncthreads();  // slots, red_m and qfrag free for the next item
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
