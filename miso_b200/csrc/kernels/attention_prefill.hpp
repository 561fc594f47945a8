#pragma once

// Drop-in CUDA (sm_100a) counterpart of the reference header kernels/attention_prefill.hpp:
// gated full attention for n consecutive tokens at positions pos0 .. pos0 + n - 1.
//   attn_prep_batch: the decode prep (norms, RoPE, KV append) for all n x 18 heads.
//   attn_prefill:    causal attention, one work item per (4-token block, KV head).
// Names, Params and launch conventions follow the reference (kernels/attention_prefill.hpp
// :20-161); the bodies are written for 32-lane CUDA warps. The tensor-core prefill with
// its own geometry is miso_attn_prefill_tc() in include/miso_cuda.h.

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
// [4b, 4b + 4), and token t sees keys [0, pos0 + t].
//
// Tensor-core body inside the caller's geometry (kBlock = 256 threads = 8 warps, no dynamic shared
// memory), the split-K decode body of attention_decode.hpp applied per token: warp w serves token
// w % 4 of the block (its 8 query heads) over the 16-key slabs s = w / 4, w / 4 + 2, ... of its
// causal range, so the two warps of a token take the even and the odd slabs and the four warps of
// one parity read the same slab at the same time (one L1 fill serves all four). Per slab:
//   S^T[16 keys][8 heads] = K Q^T and O^T[256 dims][8 heads] += V^T P^T on mma.sync m16n8k16,
//   K and V streamed from global memory into fragments (the next slab's loads in flight while the
//   current one is computed), the fp32 query and the probabilities split into fp16 high and low
//   parts (two MMAs each; K and V are exact fp16), so the result keeps fp32 accuracy.
// A warp visits only slabs that hold at least one key its token sees and masks the keys past it,
// so a token's result does not depend on the block it shares or on how the prompt was cut into
// calls. The two warp states of a token are merged through shared memory (the query fragments'
// space) and the gated output is written by the even warp.
template <int kBlock>
__device__ void attn_prefill_op(const AttnPrefillParams& p, unsigned first, unsigned count) {
  using namespace attn;
  using attn_detail::kSplitSlotFloats;
  using attn_detail::kSplitSlotHead;
  using attn_detail::split_slot_index;
  constexpr int kGroup = kQHeads / kKvHeads, kQB = kAttnQBlock, kSlab = 16;
  static_assert(kBlock == 2 * kQB * kWave && kWave == 32 && kGroup == 8, "two warps per token");
  // Query fragments per token, k-step and lane: {hi b0, hi b1, lo b0, lo b1}.
  constexpr int kQfragBytes = kQB * 16 * 32 * 16;
  constexpr int kSlotBytes = kQB * kSplitSlotFloats * 4;
  __shared__ __align__(16) unsigned char smem[kQfragBytes > kSlotBytes ? kQfragBytes : kSlotBytes];
  __shared__ float red_m[2 * kQB][kGroup];
  auto qfrag = reinterpret_cast<uint4(*)[16][32]>(smem);
  auto slot = reinterpret_cast<float(*)[kSplitSlotFloats]>(smem);
  const unsigned tid = threadIdx.x, warp = tid / kWave, lane = tid % kWave;
  const unsigned r = warp % kQB, parity = warp / kQB;
  const unsigned g = lane / 4, tq = lane % 4;
  const float kNegInf = -__int_as_float(0x7f800000);
  auto word = [](const uint4& v, int i) -> uint32_t {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
  };

  for (unsigned item = first + blockIdx.x; item < first + count; item += gridDim.x) {
    const unsigned kvh = item % kKvHeads, t0 = item / kKvHeads * kQB;
    const unsigned nq = min(static_cast<unsigned>(kQB), p.n - t0);
    const half_t* K = p.k_cache + std::size_t{kvh} * p.max_ctx * kDim;
    const half_t* V = p.v_cache + std::size_t{kvh} * p.max_ctx * kDim;

    // Q^T fragments of each token's 8 heads (pre-scaled by 1/16 = 1/sqrt(256), exact): k-step
    // ks, lane (fg, ft) holds dims 64 ft + 4 ks + {0, 1} (b0) and + {2, 3} (b1) of head fg.
    for (unsigned e = tid; e < kQB * 16 * 32; e += kBlock) {
      const unsigned tr = e / 512, ks = e / 32 % 16, ln = e % 32, fg = ln / 4, ft = ln % 4;
      uint4 f = make_uint4(0, 0, 0, 0);
      if (tr < nq) {
        const float4 x = *reinterpret_cast<const float4*>(
            p.q + (std::size_t{t0 + tr} * kQHeads + kvh * kGroup + fg) * kDim + 64 * ft + 4 * ks);
        dev::split_half2(x.x * 0.0625f, x.y * 0.0625f, f.x, f.z);
        dev::split_half2(x.z * 0.0625f, x.w * 0.0625f, f.y, f.w);
      }
      qfrag[tr][ks][ln] = f;
    }
    __syncthreads();

    const unsigned j_end = p.pos0 + t0 + r + 1;  // keys [0, j_end) of this warp's token
    const unsigned nslab = r < nq ? (j_end + kSlab - 1) / kSlab : 0;
    float o[16][4];
#pragma unroll
    for (int mb = 0; mb < 16; ++mb)
      o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.0f;
    float m0 = kNegInf, m1 = kNegInf, l0 = 0.0f, l1 = 0.0f;

    // K rows g, g + 8 of a slab: dims [64 tq, +64) as 8 x 16 bytes each; V rows 2 tq, 2 tq + 1,
    // 2 tq + 8, 2 tq + 9: dims [32 g, +32) as 4 x 16 bytes each. Keys at or past j_end are not
    // read (zero).
    uint4 kr[2][8], vr[4][4];
    auto load_k = [&](unsigned s) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const unsigned key = kSlab * s + g + 8 * h;
        const uint4* row = reinterpret_cast<const uint4*>(K + std::size_t{key} * kDim + 64 * tq);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          kr[h][c] = key < j_end ? __ldg(row + c) : make_uint4(0, 0, 0, 0);
      }
    };
    auto load_v = [&](unsigned s) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const unsigned key = kSlab * s + 2 * tq + (h & 1) + 8 * (h >> 1);
        const uint4* row = reinterpret_cast<const uint4*>(V + std::size_t{key} * kDim + 32 * g);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          vr[h][c] = key < j_end ? __ldg(row + c) : make_uint4(0, 0, 0, 0);
      }
    };

    if (parity < nslab) {
      load_k(parity);
      load_v(parity);
    }
    for (unsigned s = parity; s < nslab; s += 2) {
      const unsigned key0 = kSlab * s;
      // ---- S^T = K Q^T (hi and lo query parts in separate accumulators) ----------------------
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 16; ++ks) {
        const uint32_t a0 = word(kr[0][ks / 2], 2 * (ks % 2));
        const uint32_t a2 = word(kr[0][ks / 2], 2 * (ks % 2) + 1);
        const uint32_t a1 = word(kr[1][ks / 2], 2 * (ks % 2));
        const uint32_t a3 = word(kr[1][ks / 2], 2 * (ks % 2) + 1);
        const uint4 qf = qfrag[r][ks][lane];
        dev::mma_f16(sa, a0, a1, a2, a3, qf.x, qf.y);
        dev::mma_f16(sb, a0, a1, a2, a3, qf.z, qf.w);
      }
      if (s + 2 < nslab)
        load_k(s + 2);  // the K registers are free: start the next slab's keys
      float sv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        sv[i] = sa[i] + sb[i];
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
      if (s + 2 < nslab)
        load_v(s + 2);
    }

    // ---- merge the two warp states of each token, then the gated output ----------------------
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (g == 0)
      red_m[warp][2 * tq] = m0, red_m[warp][2 * tq + 1] = m1;
    __syncthreads();  // every warp is past its last query-fragment read: the slots may reuse it
    const float M0 = fmaxf(m0, red_m[warp ^ kQB][2 * tq]);
    const float M1 = fmaxf(m1, red_m[warp ^ kQB][2 * tq + 1]);
    const float sc0 = m0 == kNegInf ? 0.0f : __expf(m0 - M0);  // the odd warp may have no keys
    const float sc1 = m1 == kNegInf ? 0.0f : __expf(m1 - M1);
    l0 *= sc0, l1 *= sc1;
#pragma unroll
    for (int mb = 0; mb < 16; ++mb)
      o[mb][0] *= sc0, o[mb][1] *= sc1, o[mb][2] *= sc0, o[mb][3] *= sc1;
    float* sl = slot[r];
    if (parity == 1 && r < nq) {
#pragma unroll
      for (int mb = 0; mb < 16; ++mb) {
        const unsigned d = 32 * g + 2 * mb;
        sl[split_slot_index(2 * tq, d)] = o[mb][0];
        sl[split_slot_index(2 * tq + 1, d)] = o[mb][1];
        sl[split_slot_index(2 * tq, d + 1)] = o[mb][2];
        sl[split_slot_index(2 * tq + 1, d + 1)] = o[mb][3];
      }
      if (g == 0)
        sl[8 * kSplitSlotHead + 2 * tq] = l0, sl[8 * kSplitSlotHead + 2 * tq + 1] = l1;
    }
    __syncthreads();
    if (parity == 0 && r < nq) {
      // Each lane adds the odd warp's values at the slot indices it then overwrites.
#pragma unroll
      for (int mb = 0; mb < 16; ++mb) {
        const unsigned d = 32 * g + 2 * mb;
        const int i0 = split_slot_index(2 * tq, d), i1 = split_slot_index(2 * tq + 1, d);
        const int i2 = split_slot_index(2 * tq, d + 1), i3 = split_slot_index(2 * tq + 1, d + 1);
        sl[i0] = o[mb][0] + sl[i0];
        sl[i1] = o[mb][1] + sl[i1];
        sl[i2] = o[mb][2] + sl[i2];
        sl[i3] = o[mb][3] + sl[i3];
      }
      __syncwarp();  // l of every head is complete before the g == 0 lanes update it
      if (g == 0) {
        sl[8 * kSplitSlotHead + 2 * tq] += l0;
        sl[8 * kSplitSlotHead + 2 * tq + 1] += l1;
      }
      __syncwarp();
      const unsigned t = t0 + r;
      for (unsigned h = 0; h < static_cast<unsigned>(kGroup); ++h) {
        const unsigned head = kvh * kGroup + h;
        const float L = sl[8 * kSplitSlotHead + h];
        const float* gate = p.qg + std::size_t{t} * p.qg_stride + head * 2 * kDim + kDim;
        float* out = p.core + (std::size_t{t} * kQHeads + head) * kDim;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const unsigned d = 32 * c + lane;
          out[d] = sl[split_slot_index(h, d)] / L / (1.0f + __expf(-gate[d]));
        }
      }
    }
    __syncthreads();  // slots and red_m free for the next item
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) attn_prefill_kernel(AttnPrefillParams p) {
  attn_prefill_op<kBlock>(p, 0, attn_prefill_items(p.n));
}

}  // namespace miso::kernels
