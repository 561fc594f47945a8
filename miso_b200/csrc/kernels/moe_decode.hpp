#pragma once

// Sparse MoE block of one token (256 experts, top 8, plus the shared expert), the drop-in for the
// reference's kernels/moe_decode.hpp (interface :27-31, :159-169, :219-229; launched by
// src/engine/moe.hip:56-79). Three launches:
//   moe_router:  logits[257] = W_r x with BF16 router rows (rows 0..255 the experts, row 256 the
//                shared-expert gate).
//   moe_gate_up: every block re-derives the top 8 of logits[0..255] (ties to the lower index;
//                weights = softmax of the 8 selected logits, i.e. the 256-way softmax renormalised
//                over the 8), block 0 publishes ids / weights, and warps compute
//                h[slot][r] = SiLU(gate_e[r] . x) * (up_e[r] . x) for the 8 slots and the shared
//                expert (slot 8), Q4_K r1 rows, K = 2048.
//   moe_down:    out[r] = sum_k w_k down_{e_k}[r] . h_k + sigmoid(logits[256]) down_sh[r] . h_8,
//                Q4_K or Q6_K r1 rows, K = 512.
// Activations of the GEMV products are FP16-rounded (x for gate / up, h for down), products
// accumulate in FP32 (gemv_common.hpp).

#include <cstddef>
#include <cstdint>

#include "gemv_common.hpp"

namespace miso::kernels {

namespace moe {
inline constexpr unsigned kExperts = 256;
inline constexpr unsigned kTopK = 8;
inline constexpr unsigned kSlots = 9;  // top 8 + the shared expert
inline constexpr unsigned kHidden = 2048;
inline constexpr unsigned kFf = 512;  // rows of gate / up, K of down
}  // namespace moe

struct MoeRouterParams {
  const std::uint16_t* w;  // [257][2048] BF16: 256 router rows, then the shared-expert gate
  const float* x;          // [2048]
  float* logits;           // [257]
};

namespace moe_detail {

// One router row against x, one warp: lane l takes the 8-element groups l + 32 i (i < 8), so the
// warp's loads are contiguous, then the warp sums. The batched router calls the same function,
// so decode and prefill logits are bitwise equal and route identically.
__device__ inline float router_row(const std::uint16_t* row, const float* x) {
  const unsigned lane = threadIdx.x % kWave;
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const unsigned g = lane + 32 * i;
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(row) + g);
    const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * g);
    const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * g + 1);
    acc += __uint_as_float(w.x << 16) * a.x + __uint_as_float(w.x & 0xFFFF0000u) * a.y +
           __uint_as_float(w.y << 16) * a.z + __uint_as_float(w.y & 0xFFFF0000u) * a.w +
           __uint_as_float(w.z << 16) * b.x + __uint_as_float(w.z & 0xFFFF0000u) * b.y +
           __uint_as_float(w.w << 16) * b.z + __uint_as_float(w.w & 0xFFFF0000u) * b.w;
  }
  return wave_sum(acc);
}

// Top 8 of logits[0..255] by one warp: value descending, the lower index first among equal
// values. weights[k] = exp(l_k - l_0) / sum_j exp(l_j - l_0). Every lane returns the same ids /
// weights.
__device__ inline void topk(const float* logits, int (&ids)[moe::kTopK],
                            float (&weights)[moe::kTopK]) {
  const unsigned lane = threadIdx.x % kWave;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    v[j] = logits[lane + 32 * j];
  unsigned taken = 0;
  float sel[moe::kTopK];
#pragma unroll
  for (unsigned k = 0; k < moe::kTopK; ++k) {
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // ascending index: the first strict maximum is the lowest
      const int idx = static_cast<int>(lane + 32 * j);
      if (!(taken >> j & 1u) && (v[j] > bv || bi == 0x7FFFFFFF))
        bv = v[j], bi = idx;
    }
#pragma unroll
    for (int off = kWave / 2; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi))
        bv = ov, bi = oi;
    }
    ids[k] = bi, sel[k] = bv;
    if (static_cast<unsigned>(bi) % 32 == lane)
      taken |= 1u << (bi / 32);
  }
  float z = 0.0f;
#pragma unroll
  for (unsigned k = 0; k < moe::kTopK; ++k) {
    weights[k] = expf(sel[k] - sel[0]);
    z += weights[k];
  }
#pragma unroll
  for (unsigned k = 0; k < moe::kTopK; ++k)
    weights[k] /= z;
}

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

}  // namespace moe_detail

// Router rows [first, first + count) of 257; one warp per row (grid-stride over warps).
template <int kBlock>
__device__ inline void moe_router_op(const MoeRouterParams& p, unsigned first, unsigned count) {
  constexpr unsigned kWarps = kBlock / kWave;
  for (unsigned r = first + blockIdx.x * kWarps + threadIdx.x / kWave; r < first + count;
       r += gridDim.x * kWarps) {
    const float v = moe_detail::router_row(p.w + std::size_t{r} * moe::kHidden, p.x);
    if (threadIdx.x % kWave == 0)
      p.logits[r] = v;
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) moe_router_kernel(MoeRouterParams p) {
  moe_router_op<kBlock>(p, 0, moe::kExperts + 1);
}

struct MoeGateUpParams {
  const float* logits;            // [257]
  const std::uint8_t* gate_exps;  // Q4_K r1, [256 experts][512 rows], K = 2048
  const std::uint8_t* up_exps;
  const std::uint8_t* gate_sh;  // Q4_K r1, [512 rows]
  const std::uint8_t* up_sh;
  const float* x;  // [2048]
  float* h;        // [9 slots][512]: SiLU(gate) * up; slot 8 = shared
  int* ids;        // [8], written by block 0
  float* weights;  // [8]
};

// Rows [first, first + count) of the 9 * 512 (slot-major).
template <int kBlock>
__device__ inline void moe_gate_up_op(const MoeGateUpParams& p, unsigned first, unsigned count) {
  using gemv::Fmt;
  constexpr unsigned kWarps = kBlock / kWave;
  constexpr std::size_t kRow = gemv::q4k_row_bytes(moe::kHidden);
  __shared__ gemv::StagedX<moe::kHidden> s;
  __shared__ int ids[moe::kTopK];
  if (threadIdx.x < kWave) {
    int id[moe::kTopK];
    float w[moe::kTopK];
    moe_detail::topk(p.logits, id, w);
    if (threadIdx.x < moe::kTopK) {
      ids[threadIdx.x] = id[threadIdx.x];
      if (blockIdx.x == 0)
        p.ids[threadIdx.x] = id[threadIdx.x], p.weights[threadIdx.x] = w[threadIdx.x];
    }
  }
  gemv::stage_x<Fmt::Q4K, moe::kHidden, kBlock>(p.x, s);  // ends with a barrier
  for (unsigned q = first + blockIdx.x * kWarps + threadIdx.x / kWave; q < first + count;
       q += gridDim.x * kWarps) {
    const unsigned slot = q / moe::kFf, r = q % moe::kFf;
    const std::size_t row =
        slot < moe::kTopK ? std::size_t{static_cast<unsigned>(ids[slot])} * moe::kFf + r : r;
    const std::uint8_t* g = (slot < moe::kTopK ? p.gate_exps : p.gate_sh) + row * kRow;
    const std::uint8_t* u = (slot < moe::kTopK ? p.up_exps : p.up_sh) + row * kRow;
    const float gv = wave_sum(gemv::row_partial<Fmt::Q4K, moe::kHidden>(g, s));
    const float uv = wave_sum(gemv::row_partial<Fmt::Q4K, moe::kHidden>(u, s));
    if (threadIdx.x % kWave == 0)
      p.h[q] = moe_detail::silu(gv) * uv;
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) moe_gate_up_kernel(MoeGateUpParams p) {
  moe_gate_up_op<kBlock>(p, 0, moe::kSlots * moe::kFf);
}

enum class QType { Q4K, Q6K };

struct MoeDownParams {
  const float* logits;            // [257]; logits[256] gates the shared expert
  const int* ids;                 // [8]
  const float* weights;           // [8]
  const std::uint8_t* down_exps;  // r1, [256 experts][2048 rows], K = 512
  const std::uint8_t* down_sh;    // r1, [2048 rows]
  const float* h;                 // [9][512] SiLU(gate) * up from moe_gate_up
  float* out;                     // [2048]
};

namespace moe_detail {
template <QType T>
inline constexpr gemv::Fmt fmt_of = T == QType::Q4K ? gemv::Fmt::Q4K : gemv::Fmt::Q6K;
}  // namespace moe_detail

// Output rows [first, first + count) of 2048, one warp per row: lanes 0..15 take slot 2 i,
// lanes 16..31 slot 2 i + 1 (i < 5), each lane one 32-weight chunk of the K = 512 row.
template <QType T, int kBlock>
__device__ inline void moe_down_op(const MoeDownParams& p, unsigned first, unsigned count) {
  constexpr gemv::Fmt F = moe_detail::fmt_of<T>;
  constexpr unsigned kWarps = kBlock / kWave, K = moe::kFf;
  constexpr std::size_t kRow = gemv::row_bytes<F>(K);
  static_assert(K / 32 == kWave / 2, "half a warp covers one K = 512 row");
  __shared__ gemv::StagedX<K> s[moe::kSlots];
  __shared__ float w[moe::kSlots];
  __shared__ int ids[moe::kTopK];
  if (threadIdx.x < moe::kTopK)
    w[threadIdx.x] = p.weights[threadIdx.x], ids[threadIdx.x] = p.ids[threadIdx.x];
  if (threadIdx.x == 0)
    w[moe::kTopK] = moe_detail::sigmoid(p.logits[moe::kExperts]);
  for (unsigned k = 0; k < moe::kSlots; ++k)
    gemv::stage_x<F, K, kBlock>(p.h + k * K, s[k]);  // each ends with a barrier
  const unsigned lane = threadIdx.x % kWave, half = lane / 16, c = lane % 16;
  for (unsigned r = first + blockIdx.x * kWarps + threadIdx.x / kWave; r < first + count;
       r += gridDim.x * kWarps) {
    float acc = 0.0f;
#pragma unroll
    for (unsigned i = 0; i < (moe::kSlots + 1) / 2; ++i) {
      const unsigned slot = 2 * i + half;
      if (slot < moe::kSlots) {
        const std::uint8_t* row =
            slot < moe::kTopK
                ? p.down_exps + (std::size_t{static_cast<unsigned>(ids[slot])} * moe::kHidden + r) * kRow
                : p.down_sh + std::size_t{r} * kRow;
        acc += w[slot] * gemv::chunk_dot<F, K>(gemv::load_chunk<F>(row, K, c), s[slot], c);
      }
    }
    acc = wave_sum(acc);
    if (lane == 0)
      p.out[r] = acc;
  }
}

template <QType T, int kBlock>
__global__ void __launch_bounds__(kBlock) moe_down_kernel(MoeDownParams p) {
  moe_down_op<T, kBlock>(p, 0, moe::kHidden);
}

}  // namespace miso::kernels
