#pragma once

// Token embedding lookup from a Q4_K r1 table: out[t] = dequant(table[ids[t]]) — the drop-in for
// the reference's kernels/embed.hpp (interface :13-17, :44-47; launched by src/engine/model.hip:
// 109-110, 141-142 as embed_q4k_kernel<2048, 256><<<tokens, 256>>>). Bit-exact with a CPU
// dequantisation: d * sc, (d * sc) * q and dmin * m are exact in FP32 (11 + 6 + 4 significant
// bits at most), so the one rounding is the subtraction, done here without contraction.
//
// One block per token; thread i expands the 16 weights of 16-byte nibble chunk i (low or high
// nibbles of half a group) and writes them as four float4.

#include <cstddef>
#include <cstdint>

#include "gemv_common.hpp"

namespace miso::kernels {

struct EmbedParams {
  const std::uint8_t* table;  // vocab rows of kN / 256 Q4_K r1 blocks
  const std::int32_t* ids;    // [tokens]
  float* out;                 // [tokens][kN]
};

// Tokens [first, first + count); one block per token (grid-stride).
template <unsigned kN, int kBlock>
__device__ inline void embed_q4k_op(const EmbedParams& p, unsigned first, unsigned count) {
  static_assert(kN % 256 == 0);
  constexpr unsigned kRowBytes = kN / 256 * 144;
  constexpr unsigned kUnits = kN / 16;  // (chunk, nibble half) pairs of 16 weights
  for (unsigned t = first + blockIdx.x; t < first + count; t += gridDim.x) {
    const std::uint8_t* row = p.table + std::size_t(p.ids[t]) * kRowBytes;
    float* out = p.out + std::size_t{t} * kN;
    for (unsigned u = threadIdx.x; u < kUnits; u += kBlock) {
      const unsigned c = u / 2, hi = u % 2, b = c / 8, j = c % 8, g = j / 2;
      const std::uint8_t* blk = row + std::size_t{b} * 144;
      const uint4 h = __ldg(reinterpret_cast<const uint4*>(blk));
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * j));
      const unsigned bit = 24 * g;
      const uint32_t lo_w = gemv::word(h, 1 + bit / 32);
      const uint32_t hi_w = bit / 32 + 2 < 4 ? gemv::word(h, 2 + bit / 32) : 0u;
      const uint32_t f = __funnelshift_r(lo_w, hi_w, bit % 32) >> (12 * hi);
      const float dsc = __fmul_rn(gemv::f16_bits(h.x & 0xFFFFu), gemv::small_int_f(f & 63u));
      const float dm = __fmul_rn(gemv::f16_bits(h.x >> 16), gemv::small_int_f((f >> 6) & 63u));
      float4* dst = reinterpret_cast<float4*>(out + gemv::chunk_elem<gemv::Fmt::Q4K>(c, hi, 0));
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint32_t wd = gemv::word(q, v);
        float r[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          r[e] = __fsub_rn(__fmul_rn(dsc, gemv::small_int_f((wd >> (8 * e + 4 * hi)) & 15u)), dm);
        dst[v] = make_float4(r[0], r[1], r[2], r[3]);
      }
    }
  }
}

template <unsigned kN, int kBlock>
__global__ void __launch_bounds__(kBlock) embed_q4k_kernel(EmbedParams p, unsigned tokens) {
  embed_q4k_op<kN, kBlock>(p, 0, tokens);
}

}  // namespace miso::kernels
