#pragma once

// Residual add + RMSNorm, the drop-in for the reference's kernels/rmsnorm.hpp (interface
// :17-25, launch add_rmsnorm_kernel<kN, kRmsNormBlock><<<tokens, kRmsNormBlock>>> as in
// src/engine/attention.hip:82-85, model.hip:92-94):
//   residual += delta (when delta is not null);  out = residual * rsqrt(mean(residual^2) + eps) * w.
// The weight tensor of the GGUF already holds 1 + w, so it multiplies directly.
//
// CUDA layout: one block per token (grid-stride over tokens); each thread owns kN / (4 kBlock)
// float4 vectors, so every load and store is a coalesced 16-byte access; the sum of squares is a
// warp butterfly followed by one shared-memory pass over the block's warps.

#include <cstddef>

#include "wave.hpp"

namespace miso::kernels {

// Threads per token. 2048 / 256 = 8 floats (two float4) per thread.
inline constexpr int kRmsNormBlock = 256;

struct AddRmsNormParams {
  float* residual;      // [tokens][kN], updated in place when delta is not null
  const float* delta;   // [tokens][kN], or nullptr for a plain RMSNorm
  const float* weight;  // [kN]
  float* out;           // [tokens][kN]
  float eps;
};

// Tokens [first, first + count).
template <unsigned kN, int kBlock>
__device__ inline void add_rmsnorm_op(const AddRmsNormParams& p, unsigned first, unsigned count) {
  static_assert(kN % (4 * kBlock) == 0, "each thread owns whole float4 vectors");
  constexpr int kVec = kN / (4 * kBlock);
  __shared__ float scratch[kBlock / kWave];
  for (unsigned t = first + blockIdx.x; t < first + count; t += gridDim.x) {
    float4* res = reinterpret_cast<float4*>(p.residual + std::size_t{t} * kN);
    const float4* del =
        p.delta != nullptr ? reinterpret_cast<const float4*>(p.delta + std::size_t{t} * kN) : nullptr;
    float4 h[kVec];
    float ss = 0.0f;
#pragma unroll
    for (int v = 0; v < kVec; ++v) {
      const unsigned i = threadIdx.x + v * kBlock;
      h[v] = res[i];
      if (del != nullptr) {
        const float4 d = del[i];
        h[v].x += d.x, h[v].y += d.y, h[v].z += d.z, h[v].w += d.w;
      }
      ss += h[v].x * h[v].x + h[v].y * h[v].y + h[v].z * h[v].z + h[v].w * h[v].w;
    }
    const float r = rsqrtf(block_sum<kBlock>(ss, scratch) / static_cast<float>(kN) + p.eps);
    const float4* w = reinterpret_cast<const float4*>(p.weight);
    float4* out = reinterpret_cast<float4*>(p.out + std::size_t{t} * kN);
#pragma unroll
    for (int v = 0; v < kVec; ++v) {
      const unsigned i = threadIdx.x + v * kBlock;
      if (del != nullptr)
        res[i] = h[v];
      const float4 g = w[i];
      out[i] = make_float4(h[v].x * r * g.x, h[v].y * r * g.y, h[v].z * r * g.z, h[v].w * r * g.w);
    }
  }
}

template <unsigned kN, int kBlock>
__global__ void __launch_bounds__(kBlock) add_rmsnorm_kernel(AddRmsNormParams p, unsigned tokens) {
  add_rmsnorm_op<kN, kBlock>(p, 0, tokens);
}

}  // namespace miso::kernels
