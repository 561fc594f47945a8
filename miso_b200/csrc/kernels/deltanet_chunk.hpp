#pragma once

// Drop-in CUDA (sm_100a) counterpart of the reference header kernels/deltanet_chunk.hpp: prefill
// Gated DeltaNet as a batched conv, a norm pass and the chunked gated delta rule (chunk 64).
//
// The recurrence per V head is the one of deltanet_step.hpp. Over a chunk of C tokens, with
// g_t = sum_{i<=t} log(alpha_i) inside the chunk (reference formulas, kernels/deltanet_chunk.hpp
// :3-9):
//   (I + L) delta = beta (v - e^g (S^T k)),   L[t][j] = beta_t e^(g_t - g_j) (k_j . k_t), j < t
//   o_t = e^(g_t) (S^T q_t) + sum_{j<=t} e^(g_t - g_j) (k_j . q_t) delta_j
//   S   = e^(g_last) S + sum_j e^(g_last - g_j) k_j delta_j^T
// Conv, SiLU and the q / k L2 norms match deltanet_seq_op, so states and outputs agree with the
// token recurrence up to reassociation.

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "deltanet_step.hpp"
#include "wave.hpp"

namespace miso::kernels {

constexpr unsigned kDeltaChunk = 64;

struct DeltaNetConvParams {
  const float* qkv;  // [n][8192]
  const float* a;    // [n][32]
  const float* b;    // [n][32]
  const float* conv_w;
  const float* conv_in;
  float* conv_out;
  const float* ssm_a;
  const float* dt_bias;
  float* q;      // [n][16][128] normalised
  float* k;      // [n][16][128]
  float* v;      // [n][32][128]
  float* beta;   // [n][32]
  float* log_a;  // [n][32] log(alpha)
  unsigned n;
};

// Channels [first, first + count) of 8192; one thread walks every token of one channel, writing
// the SiLU'd conv output (q / k raw, normalised later by deltanet_norm_op) and the final history.
__device__ inline void deltanet_conv_op(const DeltaNetConvParams& p, unsigned first,
                                        unsigned count) {
  using namespace deltanet_detail;
  constexpr unsigned kQk = kKHeads * kDim, kCh = 2 * kQk + kVHeads * kDim;
  for (unsigned c = first + blockIdx.x * blockDim.x + threadIdx.x; c < first + count;
       c += gridDim.x * blockDim.x) {
    const float w0 = p.conv_w[4 * c], w1 = p.conv_w[4 * c + 1], w2 = p.conv_w[4 * c + 2],
                w3 = p.conv_w[4 * c + 3];
    float h0 = p.conv_in[3 * c], h1 = p.conv_in[3 * c + 1], h2 = p.conv_in[3 * c + 2];
    float* dst;
    std::size_t stride;
    if (c < kQk) {
      dst = p.q + c, stride = kQk;
    } else if (c < 2 * kQk) {
      dst = p.k + (c - kQk), stride = kQk;
    } else {
      dst = p.v + (c - 2 * kQk), stride = kVHeads * kDim;
    }
    for (unsigned tok = 0; tok < p.n; ++tok) {
      const float x = p.qkv[std::size_t{tok} * kCh + c];
      dst[std::size_t{tok} * stride] = silu(w0 * h0 + w1 * h1 + w2 * h2 + w3 * x);
      h0 = h1, h1 = h2, h2 = x;
    }
    p.conv_out[3 * c] = h0;
    p.conv_out[3 * c + 1] = h1;
    p.conv_out[3 * c + 2] = h2;
  }
}

__global__ void __launch_bounds__(256) deltanet_conv_kernel(DeltaNetConvParams p) {
  using namespace deltanet_detail;
  deltanet_conv_op(p, 0, kKHeads * kDim * 2 + kVHeads * kDim);
}

// Items [first, first + count): [0, 16) q heads, [16, 32) k heads (L2 norm in place, q also
// scaled by 1/sqrt(128)), [32, 64) the beta / log(alpha) of V head item - 32. Each warp of the
// block normalises whole 128-wide rows (one token at a time, four floats per lane).
__device__ inline void deltanet_norm_op(const DeltaNetConvParams& p, unsigned first,
                                        unsigned count) {
  using namespace deltanet_detail;
  const unsigned lane = threadIdx.x % kWave, warp = threadIdx.x / kWave;
  const unsigned warps = blockDim.x / kWave;
  for (unsigned item = first + blockIdx.x; item < first + count; item += gridDim.x) {
    if (item < 2 * kKHeads) {
      const bool is_q = item < kKHeads;
      float* base = (is_q ? p.q : p.k) + (item % kKHeads) * kDim;
      for (unsigned tok = warp; tok < p.n; tok += warps) {
        float4* row = reinterpret_cast<float4*>(base + std::size_t{tok} * kKHeads * kDim);
        float4 x = row[lane];
        const float ss = wave_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
        const float r = rsqrtf(ss + 1e-6f);
        x.x *= r, x.y *= r, x.z *= r, x.w *= r;
        if (is_q) {
          const float qs = rsqrtf(static_cast<float>(kDim));
          x.x *= qs, x.y *= qs, x.z *= qs, x.w *= qs;
        }
        row[lane] = x;
      }
    } else {
      const unsigned h = item - 2 * kKHeads;
      for (unsigned tok = threadIdx.x; tok < p.n; tok += blockDim.x) {
        const std::size_t i = std::size_t{tok} * kVHeads + h;
        p.beta[i] = 1.0f / (1.0f + __expf(-p.b[i]));
        p.log_a[i] = p.ssm_a[h] * softplus(p.a[i] + p.dt_bias[h]);
      }
    }
  }
}

__global__ void __launch_bounds__(256) deltanet_norm_kernel(DeltaNetConvParams p) {
  deltanet_norm_op(p, 0, deltanet_detail::kKHeads * 2 + deltanet_detail::kVHeads);
}

struct DeltaNetChunkParams {
  const float* q;      // [n][16][128]
  const float* k;      // [n][16][128]
  const float* v;      // [n][32][128]
  const float* beta;   // [n][32]
  const float* log_a;  // [n][32]
  const float* z;      // [n][4096]
  const float* norm_w;
  float* state;  // [32][128][128]
  float* out;    // [n][4096]
  float* sk;     // [32][64][128] scratch
  float* sq;     // [32][64][128]
  unsigned n;
  float eps;
};

// V heads [first, first + count), one 256-thread block per head; chunks of 64 in order. Thread t
// holds state column t % 128, rows [64 (t / 128), +64) in registers. The per-column steps
// (forward substitution, outputs) run on threads 0..127 with no barriers, since column vi only
// needs column vi of earlier deltas; delta_i overwrites S^T k_i in sk, o_i overwrites S^T q_i in sq.
template <int kBlock>
__device__ void deltanet_chunk_op(const DeltaNetChunkParams& p, unsigned first, unsigned count) {
  using namespace deltanet_detail;
  static_assert(kBlock == 2 * kDim, "two threads per state column");
  constexpr unsigned kC = kDeltaChunk, kP = kC + 1, kR = kDim / 2;
  constexpr unsigned kKRow = kKHeads * kDim, kVRow = kVHeads * kDim;
  __shared__ float A[kC * kP];  // k_i . k_j, then L
  __shared__ float B[kC * kP];  // q_i . k_j, then decayed (j <= i)
  __shared__ float part[2][8][kDim];
  __shared__ float g[kC], beta[kC], eg[kC];
  const unsigned t = threadIdx.x, vi = t % kDim, hf = t / kDim, lane = t % kWave,
                 warp = t / kWave;

  for (unsigned h = first + blockIdx.x; h < first + count; h += gridDim.x) {
    const unsigned kh = h % kKHeads;
    float* S = p.state + std::size_t{h} * kDim * kDim;
    float s[kR];
#pragma unroll
    for (unsigned r = 0; r < kR; ++r)
      s[r] = S[(hf * kR + r) * kDim + vi];
    float* sk = p.sk + std::size_t{h} * kC * kDim;
    float* sq = p.sq + std::size_t{h} * kC * kDim;

    for (unsigned t0 = 0; t0 < p.n; t0 += kC) {
      const unsigned C = min(kC, p.n - t0);
      const float* kr = p.k + (std::size_t{t0} * kKHeads + kh) * kDim;  // token i at + i * kKRow
      const float* qr = p.q + (std::size_t{t0} * kKHeads + kh) * kDim;
      const float* vr = p.v + (std::size_t{t0} * kVHeads + h) * kDim;  // token i at + i * kVRow
      if (t < C) {
        float acc = 0.0f;
        for (unsigned i = 0; i <= t; ++i)
          acc += p.log_a[std::size_t{t0 + i} * kVHeads + h];
        g[t] = acc;
        eg[t] = __expf(acc);
        beta[t] = p.beta[std::size_t{t0 + t} * kVHeads + h];
      }
      for (unsigned e = t; e < C * C; e += kBlock) {
        const unsigned i = e / C, j = e % C;
        if (j <= i) {
          const float4* ki = reinterpret_cast<const float4*>(kr + i * kKRow);
          const float4* kj = reinterpret_cast<const float4*>(kr + j * kKRow);
          const float4* qi = reinterpret_cast<const float4*>(qr + i * kKRow);
          float dk = 0.0f, dq = 0.0f;
#pragma unroll 4
          for (unsigned c = 0; c < kDim / 4; ++c) {
            const float4 b4 = kj[c], a4 = ki[c], q4 = qi[c];
            dk += a4.x * b4.x + a4.y * b4.y + a4.z * b4.z + a4.w * b4.w;
            dq += q4.x * b4.x + q4.y * b4.y + q4.z * b4.z + q4.w * b4.w;
          }
          A[i * kP + j] = dk;
          B[i * kP + j] = dq;
        }
      }
      // S^T k_i and S^T q_i, eight tokens per round, the two row halves summed through part[].
      for (int which = 0; which < 2; ++which) {
        const float* rows = which == 0 ? kr : qr;
        float* dst = which == 0 ? sk : sq;
        for (unsigned base = 0; base < C; base += 8) {
          const unsigned m = min(8u, C - base);
          for (unsigned u = 0; u < m; ++u) {
            const float* x = rows + (base + u) * kKRow + hf * kR;
            float acc = 0.0f;
#pragma unroll
            for (unsigned r = 0; r < kR; ++r)
              acc += s[r] * x[r];
            part[hf][u][vi] = acc;
          }
          __syncthreads();
          if (hf == 0) {
            for (unsigned u = 0; u < m; ++u)
              dst[(base + u) * kDim + vi] = part[0][u][vi] + part[1][u][vi];
          }
          __syncthreads();
        }
      }
      for (unsigned e = t; e < C * C; e += kBlock) {
        const unsigned i = e / C, j = e % C;
        if (j <= i) {
          const float dec = __expf(g[i] - g[j]);
          if (j < i)
            A[i * kP + j] = beta[i] * dec * A[i * kP + j];
          B[i * kP + j] = dec * B[i * kP + j];
        }
      }
      __syncthreads();
      if (hf == 0) {
        // Forward substitution; delta_i replaces (S^T k)_i in sk.
        for (unsigned i = 0; i < C; ++i) {
          float acc = beta[i] * (vr[std::size_t{i} * kVRow + vi] - eg[i] * sk[i * kDim + vi]);
          for (unsigned j = 0; j < i; ++j)
            acc -= A[i * kP + j] * sk[j * kDim + vi];
          sk[i * kDim + vi] = acc;
        }
        // Outputs before the norm; o_i replaces (S^T q)_i in sq.
        for (unsigned i = 0; i < C; ++i) {
          float o = eg[i] * sq[i * kDim + vi];
          for (unsigned j = 0; j <= i; ++j)
            o += B[i * kP + j] * sk[j * kDim + vi];
          sq[i * kDim + vi] = o;
        }
      }
      __syncthreads();
      // Gated RMSNorm, one token per warp at a time.
      for (unsigned i = warp; i < C; i += kBlock / kWave) {
        const float4 o = reinterpret_cast<const float4*>(sq + i * kDim)[lane];
        const float ss = wave_sum(o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w);
        const float r = rsqrtf(ss / kDim + p.eps);
        const std::size_t row = (std::size_t{t0 + i} * kVHeads + h) * kDim;
        const float4 z4 = reinterpret_cast<const float4*>(p.z + row)[lane];
        const float4 w4 = reinterpret_cast<const float4*>(p.norm_w)[lane];
        float4 y;
        y.x = o.x * r * w4.x * silu(z4.x);
        y.y = o.y * r * w4.y * silu(z4.y);
        y.z = o.z * r * w4.z * silu(z4.z);
        y.w = o.w * r * w4.w * silu(z4.w);
        reinterpret_cast<float4*>(p.out + row)[lane] = y;
      }
      // State: S = e^(g_last) S + sum_i e^(g_last - g_i) k_i delta_i^T.
      {
        const float gl = g[C - 1], el = eg[C - 1];
        float add[kR];
#pragma unroll
        for (unsigned r = 0; r < kR; ++r)
          add[r] = 0.0f;
        for (unsigned i = 0; i < C; ++i) {
          const float coef = __expf(gl - g[i]) * sk[i * kDim + vi];
          const float* x = kr + i * kKRow + hf * kR;
#pragma unroll
          for (unsigned r = 0; r < kR; ++r)
            add[r] += x[r] * coef;
        }
#pragma unroll
        for (unsigned r = 0; r < kR; ++r)
          s[r] = el * s[r] + add[r];
      }
      __syncthreads();
    }
#pragma unroll
    for (unsigned r = 0; r < kR; ++r)
      S[(hf * kR + r) * kDim + vi] = s[r];
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) deltanet_chunk_kernel(DeltaNetChunkParams p) {
  deltanet_chunk_op<kBlock>(p, 0, deltanet_detail::kVHeads);
}

}  // namespace miso::kernels
