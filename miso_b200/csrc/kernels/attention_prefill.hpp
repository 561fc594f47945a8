#pragma once

// Drop-in CUDA (sm_100a) counterpart of the reference header kernels/attention_prefill.hpp:
// gated full attention for n consecutive tokens at positions pos0 .. pos0 + n - 1.
//   attn_prep_batch: the decode prep (norms, RoPE, KV append) for all n x 18 heads.
//   attn_prefill:    causal attention, one work item per (4-token block, KV head).
// Names, Params and launch conventions follow the reference (kernels/attention_prefill.hpp
// :20-161); the bodies are written for 32-lane CUDA warps. The tensor-core prefill with
// library-chosen geometry is miso_attn_prefill_bf16() in include/miso_cuda.h.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "attention_decode.hpp"
#include "wave.hpp"

namespace miso::kernels {

// Items [first, first + count) of 18 n, token-major (item = token * 18 + head).
template <int kBlock>
__device__ void attn_prep_batch_op(const AttnPrepBatchParams& p, unsigned first, unsigned count) {
  using namespace attn;
  constexpr unsigned kHeads = kQHeads + kKvHeads;
  for (unsigned item = first + blockIdx.x; item < first + count; item += gridDim.x) {
    const unsigned t = item / kHeads, head = item % kHeads;
    AttnPrepParams tok = p.tok0;
    tok.qg += std::size_t{t} * p.proj_stride;
    tok.k += std::size_t{t} * p.proj_stride;
    tok.v += std::size_t{t} * p.proj_stride;
    tok.q += std::size_t{t} * kQHeads * kDim;
    tok.pos += t;
    attn_prep_head<kBlock>(tok, head);
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) attn_prep_batch_kernel(AttnPrepBatchParams p) {
  attn_prep_batch_op<kBlock>(p, 0, p.n * (attn::kQHeads + attn::kKvHeads));
}

struct AttnPrefillParams {
  const float* q;               // [n][16][256] normalised, rotated (unscaled)
  const float* qg;              // token-major; gate at tok * qg_stride + head * 512 + 256
  const attn::half_t* k_cache;  // [2][max_ctx][256], positions [0, pos0 + n) valid
  const attn::half_t* v_cache;
  float* core;  // [n][16][256]
  unsigned pos0, n, max_ctx;
  unsigned qg_stride;  // 8192 packed, or 9216 when q/k/v share a proj buffer
};

constexpr unsigned kAttnQBlock = 4;

__host__ __device__ inline unsigned attn_prefill_items(unsigned n) {
  return attn::kKvHeads * ((n + kAttnQBlock - 1) / kAttnQBlock);
}

// Items [first, first + count) with item = block * 2 + KV head; block b covers tokens
// [4b, 4b + 4). Token t sees keys [0, pos0 + t]. One warp per query head of the KV group, for all
// four tokens of the block. Keys are visited in 16-key sub-chunks: in the score phase lane l
// takes key l % 16 for tokens 2(l / 16) and 2(l / 16) + 1 (K row stored word-rotated so the 16
// rows read distinct banks while every lane reads the same query word); in the value phase lane
// l owns dims [8l, 8l + 8) of all four tokens and reads V straight from global memory (shared by
// the eight warps through L1). Online-softmax state is per (warp, token) and warp-uniform.
template <int kBlock>
__device__ void attn_prefill_op(const AttnPrefillParams& p, unsigned first, unsigned count) {
  using namespace attn;
  constexpr int kGroup = kQHeads / kKvHeads, kQB = kAttnQBlock, kSub = 16;
  constexpr int kQRow = kGroup * kDim + 8;  // floats per token: tokens r and r+2 16 banks apart
  constexpr int kWords = kDim / 2;          // half2 words per K row
  static_assert(kBlock == kGroup * kWave, "one warp per query head of the KV group");
  static_assert(kQB == 4 && 2 * kSub == kWave, "lane layout of the score phase");
  __shared__ float qs[kQB * kQRow];
  __shared__ uint32_t ks[kSub][kWords];
  const float kNegInf = -__int_as_float(0x7f800000);
  const unsigned tid = threadIdx.x, lane = tid % kWave, h = tid / kWave;
  const unsigned kj = lane % kSub, rp = (lane / kSub) * 2;
  const float scale = rsqrtf(static_cast<float>(kDim));

  for (unsigned item = first + blockIdx.x; item < first + count; item += gridDim.x) {
    const unsigned kvh = item % kKvHeads, t0 = item / kKvHeads * kQB;
    const unsigned nq = min(static_cast<unsigned>(kQB), p.n - t0);
    const uint32_t* K = reinterpret_cast<const uint32_t*>(p.k_cache + std::size_t{kvh} * p.max_ctx * kDim);
    const uint4* V = reinterpret_cast<const uint4*>(p.v_cache + std::size_t{kvh} * p.max_ctx * kDim);
    for (unsigned i = tid; i < kQB * kGroup * kDim; i += kBlock) {
      const unsigned r = i / (kGroup * kDim), rem = i % (kGroup * kDim);
      qs[r * kQRow + rem] =
          r < nq ? p.q[(std::size_t{t0 + r} * kQHeads + kvh * kGroup) * kDim + rem] * scale : 0.0f;
    }
    float m[kQB], l[kQB], acc[kQB][8];
#pragma unroll
    for (int r = 0; r < kQB; ++r) {
      m[r] = kNegInf, l[r] = 0.0f;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        acc[r][c] = 0.0f;
    }
    const unsigned len = p.pos0 + t0 + nq;  // keys of the block's last token
    const unsigned lim = p.pos0 + t0 + rp;  // this lane's first token sees keys <= lim
    __syncthreads();

    for (unsigned j0 = 0; j0 < len; j0 += kSub) {
      const unsigned n = min(static_cast<unsigned>(kSub), len - j0);
      for (unsigned e = tid; e < kSub * kWords; e += kBlock) {
        const unsigned r = e / kWords, c = e % kWords;
        if (r < n)
          ks[r][(c + r) % kWords] = K[std::size_t{j0 + r} * kWords + c];
      }
      __syncthreads();
      float s0 = kNegInf, s1 = kNegInf;
      if (kj < n) {
        const float* q0 = qs + rp * kQRow + h * kDim;
        const float* q1 = q0 + kQRow;
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 8
        for (unsigned e = 0; e < kWords; ++e) {
          const uint32_t w = ks[kj][(e + kj) % kWords];
          const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&w));
          a0 += q0[2 * e] * kf.x + q0[2 * e + 1] * kf.y;
          a1 += q1[2 * e] * kf.x + q1[2 * e + 1] * kf.y;
        }
        const unsigned key = j0 + kj;
        if (rp < nq && key <= lim)
          s0 = a0;
        if (rp + 1 < nq && key <= lim + 1)
          s1 = a1;
      }
      // Per-token max over the 16 keys of each half-warp, then broadcast to the whole warp.
      float mx0 = s0, mx1 = s1;
#pragma unroll
      for (int off = kSub / 2; off > 0; off >>= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      float m_new[kQB];
      m_new[0] = fmaxf(m[0], __shfl_sync(0xffffffffu, mx0, 0));
      m_new[1] = fmaxf(m[1], __shfl_sync(0xffffffffu, mx1, 0));
      m_new[2] = fmaxf(m[2], __shfl_sync(0xffffffffu, mx0, kSub));
      m_new[3] = fmaxf(m[3], __shfl_sync(0xffffffffu, mx1, kSub));
      const float mn0 = rp == 0 ? m_new[0] : m_new[2];
      const float mn1 = rp == 0 ? m_new[1] : m_new[3];
      const float p0 = s0 == kNegInf ? 0.0f : __expf(s0 - mn0);
      const float p1 = s1 == kNegInf ? 0.0f : __expf(s1 - mn1);
      float sum0 = p0, sum1 = p1;
#pragma unroll
      for (int off = kSub / 2; off > 0; off >>= 1) {
        sum0 += __shfl_xor_sync(0xffffffffu, sum0, off);
        sum1 += __shfl_xor_sync(0xffffffffu, sum1, off);
      }
      const float add[kQB] = {__shfl_sync(0xffffffffu, sum0, 0), __shfl_sync(0xffffffffu, sum1, 0),
                              __shfl_sync(0xffffffffu, sum0, kSub),
                              __shfl_sync(0xffffffffu, sum1, kSub)};
#pragma unroll
      for (int r = 0; r < kQB; ++r) {
        const float corr = m_new[r] == kNegInf ? 1.0f : __expf(m[r] - m_new[r]);
        l[r] = l[r] * corr + add[r];
        m[r] = m_new[r];
#pragma unroll
        for (int c = 0; c < 8; ++c)
          acc[r][c] *= corr;
      }
      for (unsigned j = 0; j < n; ++j) {
        const float pb[kQB] = {__shfl_sync(0xffffffffu, p0, j), __shfl_sync(0xffffffffu, p1, j),
                               __shfl_sync(0xffffffffu, p0, kSub + j),
                               __shfl_sync(0xffffffffu, p1, kSub + j)};
        const uint4 raw = __ldg(V + std::size_t{j0 + j} * (kDim / 8) + lane);
        const __half2* hv = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 vf = __half22float2(hv[c]);
#pragma unroll
          for (int r = 0; r < kQB; ++r) {
            acc[r][2 * c] += pb[r] * vf.x;
            acc[r][2 * c + 1] += pb[r] * vf.y;
          }
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < kQB; ++r) {
      if (r < static_cast<int>(nq)) {
        const unsigned head = kvh * kGroup + h;
        const float* gate = p.qg + std::size_t{t0 + r} * p.qg_stride + head * 2 * kDim + kDim;
        float* out = p.core + (std::size_t{t0 + r} * kQHeads + head) * kDim;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const unsigned d = 8 * lane + c;
          out[d] = acc[r][c] / l[r] / (1.0f + __expf(-gate[d]));
        }
      }
    }
    __syncthreads();
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) attn_prefill_kernel(AttnPrefillParams p) {
  attn_prefill_op<kBlock>(p, 0, attn_prefill_items(p.n));
}

}  // namespace miso::kernels
