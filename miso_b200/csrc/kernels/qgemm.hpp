#pragma once

// Prefill GEMM Y[t][n] = sum_k W[n][k] x[t][k] for Q4_K r1 / Q6_K r1 weights with FP16-rounded
// activations and FP32 accumulation — the drop-in for the reference's kernels/qgemm.hpp
// (interface :22-37, :58-60, :289-297; launched by src/engine/weights.hip:302-327 as
// qgemm_act_kernel<<<ceil(groups / 256), 256>>> and qgemm_kernel<F><<<qgemm_tiles(n, t), 256>>>).
//
// qgemm_act rounds the activations to FP16 once and records the sum of every 32 rounded values
// (one thread per 32-group), exactly the reference's activation format.
//
// qgemm: a block computes a 64-row x 64-token tile of Y. The K axis is walked in slabs of 64: each
// slab's weights are dequantised into shared memory as FP32 (each thread expands 16 weights that
// share one scale: d * sc * q - dmin * m for Q4_K, d * scale * (q - 32) for Q6_K), the 64 tokens'
// activations are widened to FP32 beside them, and every thread accumulates a 4 x 4 register tile
// (rows tn + 16 i, tokens tt + 16 j). Rows of the shared tiles are padded to 65 floats so the
// column reads of the inner loop are conflict-free.

#include <cuda_fp16.h>

#include <cstddef>
#include <cstdint>

#include "f16_ptr.hpp"
#include "gemv_common.hpp"

namespace miso::kernels {

enum class QFormat { Q4K, Q6K };

struct QGemmActParams {
  const float* x;  // n_tok x k
  F16Out xh;       // n_tok x k, x rounded to FP16
  float* xs;       // n_tok x k / 32, sums of the rounded values of each 32-group
  unsigned k, n_tok;
};

struct QGemmParams {
  const std::uint8_t* w;  // n_rows rows in the format's r1 layout
  F16In xh;               // n_tok x k
  const float* xs;        // n_tok x k / 32 (not needed by this implementation)
  float* y;               // n_tok rows of stride ldy
  unsigned k, n_rows, n_tok, ldy;
};

// 32-groups [first, first + count) of the n_tok * k / 32, one thread each (grid-stride).
__device__ inline void qgemm_act_op(const QGemmActParams& p, unsigned first, unsigned count) {
  for (unsigned g = first + blockIdx.x * blockDim.x + threadIdx.x; g < first + count;
       g += gridDim.x * blockDim.x) {
    const float4* x = reinterpret_cast<const float4*>(p.x + std::size_t{g} * 32);
    uint2* xh = reinterpret_cast<uint2*>(p.xh.p + std::size_t{g} * 32);
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 f = x[c];
      const __half2 a = __floats2half2_rn(f.x, f.y), b = __floats2half2_rn(f.z, f.w);
      const float2 fa = __half22float2(a), fb = __half22float2(b);
      s += fa.x + fa.y + fb.x + fb.y;
      xh[c] = make_uint2(*reinterpret_cast<const uint32_t*>(&a),
                         *reinterpret_cast<const uint32_t*>(&b));
    }
    p.xs[g] = s;
  }
}

__global__ void __launch_bounds__(256) qgemm_act_kernel(QGemmActParams p) {
  qgemm_act_op(p, 0, p.n_tok * (p.k / 32));
}

namespace qgemm_detail {

inline constexpr unsigned kBM = 64;    // tokens per tile
inline constexpr unsigned kBN = 64;    // weight rows per tile
inline constexpr unsigned kSlab = 64;  // K per shared-memory stage
inline constexpr int kThreads = 256;
inline constexpr unsigned kPad = kSlab + 1;

struct Smem {
  float w[kBN][kPad];
  float x[kBM][kPad];
};

// The 16 weights k = 64 s + 16 p + i (i < 16) of 256-block b of a row, s = slab within the block,
// p = quarter of the slab: all share one scale.
template <QFormat F>
__device__ inline void expand16(const std::uint8_t* row, unsigned k, unsigned b, unsigned s,
                                unsigned p, float (&out)[16]) {
  using gemv::f16_bits;
  using gemv::small_int_f;
  if (F == QFormat::Q4K) {
    // Slab s = nibble group g: qs bytes 32 g..32 g + 31; quarters 0, 1 are the low nibbles of
    // bytes 32 g + 16 p + i (sub-block 2g), quarters 2, 3 the high nibbles of 32 g + 16 (p - 2) + i.
    const std::uint8_t* blk = row + std::size_t{b} * 144;
    const uint4 h = __ldg(reinterpret_cast<const uint4*>(blk));
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * s + 16 * (p % 2)));
    const unsigned bit = 24 * s;
    const uint32_t lo_w = gemv::word(h, 1 + bit / 32);
    const uint32_t hi_w = bit / 32 + 2 < 4 ? gemv::word(h, 2 + bit / 32) : 0u;
    const uint32_t f = __funnelshift_r(lo_w, hi_w, bit % 32) >> (p < 2 ? 0 : 12);
    const float dsc = f16_bits(h.x & 0xFFFFu) * small_int_f(f & 63u);
    const float dm = f16_bits(h.x >> 16) * small_int_f((f >> 6) & 63u);
    const unsigned shift = p < 2 ? 0 : 4;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint32_t wd = gemv::word(q, v);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        out[4 * v + e] = __fsub_rn(__fmul_rn(dsc, small_int_f((wd >> (8 * e + shift)) & 15u)), dm);
    }
  } else {
    // Slab s covers elements 64 s..: half n = s / 2, quarter u = 2 (s % 2) + p / 2, l = 16 (p % 2)
    // + i. ql byte 64 n + 32 (u % 2) + l (nibble u / 2), qh byte 32 n + l (bits 2u), scale
    // 8 n + p % 2 + 2 u.
    const unsigned nb = k / 256, n = s / 2, u = 2 * (s % 2) + p / 2, l0 = 16 * (p % 2);
    const uint4 ql = __ldg(reinterpret_cast<const uint4*>(row + std::size_t{b} * 128 + 64 * n +
                                                          32 * (u % 2) + l0));
    const uint4 qh = __ldg(reinterpret_cast<const uint4*>(row + std::size_t{nb} * 128 + b * 64 +
                                                          32 * n + l0));
    const int8_t sc = reinterpret_cast<const int8_t*>(row + std::size_t{nb} * 192 + b * 16)
        [8 * n + p % 2 + 2 * u];
    const float d = f16_bits(*reinterpret_cast<const uint16_t*>(row + std::size_t{nb} * 208 + b * 2));
    const float ds = d * static_cast<float>(sc);
    const unsigned nib = u / 2 ? 4 : 0, hb = 2 * u;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint32_t a = gemv::word(ql, v), c = gemv::word(qh, v);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t q = ((a >> (8 * e + nib)) & 15u) | ((c >> (8 * e + hb)) & 3u) << 4;
        out[4 * v + e] = ds * gemv::q6_f(q);
      }
    }
  }
}

template <QFormat F>
__device__ inline void tile(const QGemmParams& p, Smem& sm, unsigned tile_id) {
  const unsigned row_tiles = (p.n_rows + kBN - 1) / kBN;
  const unsigned n0 = (tile_id % row_tiles) * kBN, m0 = (tile_id / row_tiles) * kBM;
  const std::size_t row_bytes =
      F == QFormat::Q4K ? gemv::q4k_row_bytes(p.k) : gemv::q6k_row_bytes(p.k);
  const unsigned tid = threadIdx.x, tn = tid % 16, tt = tid / 16;
  const unsigned lr = tid / 4, lp = tid % 4;  // loader: row / token lr, quarter lp
  float acc[4][4] = {};
  for (unsigned ks = 0; ks < p.k / kSlab; ++ks) {
    float wv[16];
    if (n0 + lr < p.n_rows) {
      expand16<F>(p.w + (n0 + lr) * row_bytes, p.k, ks / 4, ks % 4, lp, wv);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        wv[i] = 0.0f;
    }
    float xv[16];
    if (m0 + lr < p.n_tok) {
      const uint4* src = reinterpret_cast<const uint4*>(p.xh.p + std::size_t{m0 + lr} * p.k +
                                                        ks * kSlab + 16 * lp);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 v = src[h];
        const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wd[e]));
          xv[8 * h + 2 * e] = f.x, xv[8 * h + 2 * e + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        xv[i] = 0.0f;
    }
    __syncthreads();  // the previous slab's reads are done
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      sm.w[lr][16 * lp + i] = wv[i];
      sm.x[lr][16 * lp + i] = xv[i];
    }
    __syncthreads();
#pragma unroll 8
    for (unsigned kk = 0; kk < kSlab; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        a[i] = sm.w[tn + 16 * i][kk], b[i] = sm.x[tt + 16 * i][kk];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[i][j] += a[i] * b[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const unsigned t = m0 + tt + 16 * j;
    if (t >= p.n_tok)
      continue;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned n = n0 + tn + 16 * i;
      if (n < p.n_rows)
        p.y[std::size_t{t} * p.ldy + n] = acc[i][j];
    }
  }
}

}  // namespace qgemm_detail

// Tiles [first, first + count) of 64 rows x 64 tokens, row tiles fastest (grid-stride).
template <QFormat F>
__device__ inline void qgemm_op(const QGemmParams& p, unsigned first, unsigned count) {
  static_assert(qgemm_detail::kThreads == 4 * qgemm_detail::kBN, "one loader thread per quarter");
  __shared__ qgemm_detail::Smem sm;
  for (unsigned t = first + blockIdx.x; t < first + count; t += gridDim.x)
    qgemm_detail::tile<F>(p, sm, t);
}

__host__ __device__ inline unsigned qgemm_tiles(unsigned n_rows, unsigned n_tok) {
  using namespace qgemm_detail;
  return (n_rows + kBN - 1) / kBN * ((n_tok + kBM - 1) / kBM);
}

template <QFormat F>
__global__ void __launch_bounds__(qgemm_detail::kThreads, 2) qgemm_kernel(QGemmParams p) {
  qgemm_op<F>(p, 0, qgemm_tiles(p.n_rows, p.n_tok));
}

}  // namespace miso::kernels
