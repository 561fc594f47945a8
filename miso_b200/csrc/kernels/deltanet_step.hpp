#pragma once

// Drop-in CUDA (sm_100a) counterpart of the reference header kernels/deltanet_step.hpp: one decode
// step of Gated DeltaNet (qwen3_5_moe linear attention) after the in-projections, and the same
// recurrence over n tokens with the state held on chip.
//
// Per V head h (K head kh = h % 16, the tiled V-head order of the GGUF):
//   q, k, v = SiLU(conv1d_4(qkv)) restricted to head kh (q, k) and h (v)
//   q = q / (|q| sqrt(128)),  k = k / |k|            (|x| = sqrt(sum x^2 + 1e-6))
//   beta = sigmoid(b[h]),  decay = exp(ssm_a[h] * softplus(a[h] + dt_bias[h]))
//   S = decay S;  delta = beta (v - S^T k);  S += k delta^T;  o = S^T q
//   out = o * rsqrt(mean(o^2) + eps) * norm_w * SiLU(z)
// (reference formulas: kernels/deltanet_step.hpp:3-13). The conv history is double-buffered
// (conv_in -> conv_out) because V heads h and h + 16 both read K head kh's history; head h < 16
// writes the q / k channels' history, every head writes its v channels'.
//
// Layout on chip: a 256-thread block owns one V head; warp w holds state rows (k index)
// [16w, 16w + 16) and lane l holds value columns [4l, 4l + 4), i.e. 16 float4 registers per
// thread, loaded and stored as 512-byte coalesced rows. deltanet_step_op and deltanet_seq_op run
// the identical per-token arithmetic (detail::token_update), so n steps and one n-token sequence
// agree bit for bit.

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "wave.hpp"

namespace miso::kernels {

struct DeltaNetStepParams {
  const float* qkv;      // [8192] in-projection output: q[2048] k[2048] v[4096]
  const float* z;        // [4096] gate projection
  const float* a;        // [32]
  const float* b;        // [32]
  const float* conv_w;   // [8192][4], tap 3 multiplies the current input
  const float* conv_in;  // [8192][3] previous inputs, oldest first
  float* conv_out;       // [8192][3]
  const float* ssm_a;    // [32] = -exp(A_log)
  const float* dt_bias;  // [32]
  const float* norm_w;   // [128]
  float* state;          // [32][128 (k)][128 (v)]
  float* out;            // [4096]
  float eps;
};

namespace deltanet_detail {

constexpr int kKHeads = 16, kVHeads = 32, kDim = 128;

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(__expf(x)); }

// Causal 4-tap conv of channel c for the current token, then SiLU; `own` also shifts the
// history of channel c into conv_out.
__device__ __forceinline__ float conv_step(const DeltaNetStepParams& p, unsigned c, bool own) {
  const float* hist = p.conv_in + 3 * c;
  const float* w = p.conv_w + 4 * c;
  const float x = p.qkv[c];
  const float y = w[0] * hist[0] + w[1] * hist[1] + w[2] * hist[2] + w[3] * x;
  if (own) {
    p.conv_out[3 * c] = hist[1];
    p.conv_out[3 * c + 1] = hist[2];
    p.conv_out[3 * c + 2] = x;
  }
  return silu(y);
}

}  // namespace deltanet_detail

namespace dn_detail {

using deltanet_detail::kDim;

// Shared scratch of one head's token update.
struct TokenShared {
  float q[kDim], k[kDim], v[kDim];
  float part[8][kDim];
  float red[8];
};

// Everything after the conv for one token: q / k L2 norms, decay, delta rule on the register
// state s (rows 16w + i, columns 4 lane + c), gated RMSNorm. Expects sh.q / sh.k / sh.v to hold
// the SiLU'd conv outputs (written before the call, no barrier needed in between: the first
// statement is a barrier). Writes out[col] for col in [0, 128) from threads 0..127.
// beta_in / a_in are the raw b[h] / a[h] inputs of this token; norm_w_t / z_t are norm_w[t] and
// this token's gate z[t] for threads t < 128 (ignored above), passed as values so that a caller
// can load them ahead of the token.
__device__ __forceinline__ void token_update(TokenShared& sh, float4 (&s)[16], float beta_in,
                                             float a_in, float ssm_a, float dt_bias,
                                             float norm_w_t, float z_t, float eps, float* out) {
  using namespace deltanet_detail;
  const unsigned t = threadIdx.x, w = t / 32, lane = t % 32;
  __syncthreads();
  // L2 norms: warps 0-3 reduce q, warps 4-7 reduce k.
  const float x = t < kDim ? sh.q[t] : sh.k[t - kDim];
  const float ss = wave_sum(x * x);
  if (lane == 0)
    sh.red[w] = ss;
  __syncthreads();
  if (t < kDim) {
    sh.q[t] = x * rsqrtf(sh.red[0] + sh.red[1] + sh.red[2] + sh.red[3] + 1e-6f) *
              rsqrtf(static_cast<float>(kDim));
  } else {
    sh.k[t - kDim] = x * rsqrtf(sh.red[4] + sh.red[5] + sh.red[6] + sh.red[7] + 1e-6f);
  }
  __syncthreads();
  const float beta = 1.0f / (1.0f + __expf(-beta_in));
  const float decay = __expf(ssm_a * softplus(a_in + dt_bias));
  // Decay, then S^T k over this warp's 16 rows.
  float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float kk = sh.k[16 * w + i];
    s[i].x *= decay, s[i].y *= decay, s[i].z *= decay, s[i].w *= decay;
    kv.x += s[i].x * kk, kv.y += s[i].y * kk, kv.z += s[i].z * kk, kv.w += s[i].w * kk;
  }
  reinterpret_cast<float4*>(sh.part[w])[lane] = kv;
  __syncthreads();
  float4 delta;
  {
    const float4* vv = reinterpret_cast<const float4*>(sh.v);
    float4 acc = reinterpret_cast<const float4*>(sh.part[0])[lane];
#pragma unroll
    for (int r = 1; r < 8; ++r) {
      const float4 pr = reinterpret_cast<const float4*>(sh.part[r])[lane];
      acc.x += pr.x, acc.y += pr.y, acc.z += pr.z, acc.w += pr.w;
    }
    const float4 v4 = vv[lane];
    delta = make_float4((v4.x - acc.x) * beta, (v4.y - acc.y) * beta, (v4.z - acc.z) * beta,
                        (v4.w - acc.w) * beta);
  }
  __syncthreads();  // everyone has read part[] before it is reused
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float kk = sh.k[16 * w + i], qq = sh.q[16 * w + i];
    s[i].x += kk * delta.x, s[i].y += kk * delta.y, s[i].z += kk * delta.z, s[i].w += kk * delta.w;
    o.x += s[i].x * qq, o.y += s[i].y * qq, o.z += s[i].z * qq, o.w += s[i].w * qq;
  }
  reinterpret_cast<float4*>(sh.part[w])[lane] = o;
  __syncthreads();
  // Gated RMSNorm over the 128 outputs (warps 0-3, one column per thread).
  float oh = 0.0f;
  if (t < kDim) {
#pragma unroll
    for (int r = 0; r < 8; ++r)
      oh += sh.part[r][t];
  }
  const float os = wave_sum(oh * oh);
  __syncthreads();  // part[] / red[] reads done before red[] is rewritten
  if (lane == 0 && w < 4)
    sh.red[w] = os;
  __syncthreads();
  if (t < kDim) {
    const float r = rsqrtf((sh.red[0] + sh.red[1] + sh.red[2] + sh.red[3]) / kDim + eps);
    out[t] = oh * r * norm_w_t * silu(z_t);
  }
}

__device__ __forceinline__ void load_state(float4 (&s)[16], const float* S) {
  const unsigned w = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float4* src = reinterpret_cast<const float4*>(S) + (16 * w) * (kDim / 4) + lane;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    s[i] = src[i * (kDim / 4)];
}

__device__ __forceinline__ void store_state(const float4 (&s)[16], float* S) {
  const unsigned w = threadIdx.x / 32, lane = threadIdx.x % 32;
  float4* dst = reinterpret_cast<float4*>(S) + (16 * w) * (kDim / 4) + lane;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    dst[i * (kDim / 4)] = s[i];
}

}  // namespace dn_detail

// V heads [first, first + count), one 256-thread block per head (grid-stride).
template <int kBlock>
__device__ void deltanet_step_op(const DeltaNetStepParams& p, unsigned first, unsigned count) {
  using namespace deltanet_detail;
  static_assert(kBlock == 2 * kDim, "eight warps of 16 state rows each");
  __shared__ dn_detail::TokenShared sh;
  const unsigned t = threadIdx.x;
  for (unsigned h = first + blockIdx.x; h < first + count; h += gridDim.x) {
    const unsigned kh = h % kKHeads;
    const bool own_qk = h < kKHeads;
    float* S = p.state + std::size_t{h} * kDim * kDim;
    float4 s[16];
    dn_detail::load_state(s, S);
    if (t < kDim) {
      sh.q[t] = conv_step(p, kh * kDim + t, own_qk);
      sh.v[t] = conv_step(p, 2 * kKHeads * kDim + h * kDim + t, true);
    } else {
      sh.k[t - kDim] = conv_step(p, kKHeads * kDim + kh * kDim + (t - kDim), own_qk);
    }
    dn_detail::token_update(sh, s, p.b[h], p.a[h], p.ssm_a[h], p.dt_bias[h],
                            t < kDim ? p.norm_w[t] : 0.0f, t < kDim ? p.z[h * kDim + t] : 0.0f,
                            p.eps, p.out + h * kDim);
    dn_detail::store_state(s, S);
    __syncthreads();
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) deltanet_step_kernel(DeltaNetStepParams p) {
  deltanet_step_op<kBlock>(p, 0, deltanet_detail::kVHeads);
}

// The same recurrence over n consecutive tokens (prefill): the state and each thread's conv
// windows stay in registers; per token the arithmetic is that of deltanet_step_op.
struct DeltaNetSeqParams {
  const float* qkv;  // [n][qkv_stride], first 8192 columns are q/k/v
  const float* z;    // [n][zab_stride], first 4096 rows
  const float* a;    // [n][zab_stride], rows 4096..4127
  const float* b;    // [n][zab_stride], rows 4128..4159
  const float* conv_w;
  const float* conv_in;  // [8192][3] before the first token
  float* conv_out;       // [8192][3] after the last token
  const float* ssm_a;
  const float* dt_bias;
  const float* norm_w;
  float* state;
  float* out;  // [n][4096]
  unsigned n;
  float eps;
  unsigned zab_stride;  // 4160, or qkv_stride when z_ab shares the proj buffer
  unsigned qkv_stride;  // 8192, or larger when qkv shares a buffer with z_ab
};

namespace dn_detail {

// Where a sequence writes its results. state / conv: the final state (in place) and conv history
// (conv_out), or null to leave them untouched. state_ckpt / conv_ckpt: the state
// [n][32][128][128] and conv history [n][8192][3] after every token, or null. Both forms share one
// body, so checkpoints carry exactly the bits a shorter sequence would leave.
struct SeqSinks {
  float* state;
  float* conv;
  float* state_ckpt;
  float* conv_ckpt;
};

template <int kBlock>
__device__ void seq_body(const DeltaNetSeqParams& p, const SeqSinks& out, unsigned first,
                         unsigned count) {
  using namespace deltanet_detail;
  static_assert(kBlock == 2 * kDim, "eight warps of 16 state rows each");
  constexpr unsigned kOut = kVHeads * kDim;
  constexpr std::size_t kStateFloats = std::size_t{kVHeads} * kDim * kDim;
  constexpr std::size_t kConvFloats = std::size_t{3} * (2 * kKHeads + kVHeads) * kDim;
  __shared__ dn_detail::TokenShared sh;
  const unsigned t = threadIdx.x;
  for (unsigned h = first + blockIdx.x; h < first + count; h += gridDim.x) {
    const unsigned kh = h % kKHeads;
    const bool own_qk = h < kKHeads;
    // Channel c0: q (t < 128) or k (t >= 128); channel c1: v (t < 128 only).
    const unsigned c0 = t < kDim ? kh * kDim + t : kKHeads * kDim + kh * kDim + (t - kDim);
    const unsigned c1 = 2 * kKHeads * kDim + h * kDim + (t % kDim);
    float w0[4], w1[4], h0[3], h1[3];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w0[i] = p.conv_w[4 * c0 + i], w1[i] = p.conv_w[4 * c1 + i];
#pragma unroll
    for (int i = 0; i < 3; ++i)
      h0[i] = p.conv_in[3 * c0 + i], h1[i] = p.conv_in[3 * c1 + i];
    const float* S = p.state + std::size_t{h} * kDim * kDim;
    float4 s[16];
    dn_detail::load_state(s, S);
    const float nw = t < kDim ? p.norm_w[t] : 0.0f;
    const float ssm_a_h = p.ssm_a[h], dt_bias_h = p.dt_bias[h];
    // A token's own inputs (conv inputs x0 / x1, b, a and the gate z[t]) are loaded one token
    // ahead, so their memory latency overlaps the previous token's update; the arithmetic is
    // unchanged.
    float nx0 = 0.0f, nx1 = 0.0f, nb = 0.0f, na = 0.0f, nz = 0.0f;
    auto load_inputs = [&](unsigned tok) {
      const float* x = p.qkv + std::size_t{tok} * p.qkv_stride;
      const std::size_t zrow = std::size_t{tok} * p.zab_stride;
      nx0 = x[c0];
      if (t < kDim) {
        nx1 = x[c1];
        nz = p.z[zrow + h * kDim + t];
      }
      nb = p.b[zrow + h];
      na = p.a[zrow + h];
    };
    if (p.n > 0)
      load_inputs(0);
    for (unsigned tok = 0; tok < p.n; ++tok) {
      const float x0 = nx0, x1 = nx1, b_in = nb, a_in = na, z_t = nz;
      if (tok + 1 < p.n)
        load_inputs(tok + 1);
      const float y0 = silu(w0[0] * h0[0] + w0[1] * h0[1] + w0[2] * h0[2] + w0[3] * x0);
      h0[0] = h0[1], h0[1] = h0[2], h0[2] = x0;
      if (t < kDim) {
        const float y1 = silu(w1[0] * h1[0] + w1[1] * h1[1] + w1[2] * h1[2] + w1[3] * x1);
        h1[0] = h1[1], h1[1] = h1[2], h1[2] = x1;
        sh.q[t] = y0, sh.v[t] = y1;
      } else {
        sh.k[t - kDim] = y0;
      }
      dn_detail::token_update(sh, s, b_in, a_in, ssm_a_h, dt_bias_h, nw, z_t, p.eps,
                              p.out + std::size_t{tok} * kOut + h * kDim);
      if (out.state_ckpt != nullptr)
        dn_detail::store_state(s, out.state_ckpt + tok * kStateFloats + std::size_t{h} * kDim * kDim);
      if (out.conv_ckpt != nullptr) {
        float* cc = out.conv_ckpt + tok * kConvFloats;
        if (own_qk) {
#pragma unroll
          for (int i = 0; i < 3; ++i)
            cc[3 * c0 + i] = h0[i];
        }
        if (t < kDim) {
#pragma unroll
          for (int i = 0; i < 3; ++i)
            cc[3 * c1 + i] = h1[i];
        }
      }
    }
    if (out.state != nullptr)
      dn_detail::store_state(s, out.state + std::size_t{h} * kDim * kDim);
    if (out.conv != nullptr) {
      if (own_qk) {
#pragma unroll
        for (int i = 0; i < 3; ++i)
          out.conv[3 * c0 + i] = h0[i];
      }
      if (t < kDim) {
#pragma unroll
        for (int i = 0; i < 3; ++i)
          out.conv[3 * c1 + i] = h1[i];
      }
    }
    __syncthreads();
  }
}

}  // namespace dn_detail

template <int kBlock>
__device__ void deltanet_seq_op(const DeltaNetSeqParams& p, unsigned first, unsigned count) {
  dn_detail::seq_body<kBlock>(p, {p.state, p.conv_out, nullptr, nullptr}, first, count);
}

// Speculative verification (multi-token prediction): the same n-token recurrence and outputs as
// deltanet_seq_op, but p.state and p.conv_out are left untouched; the state and conv history
// after every token go to state_ckpt [n][32][128][128] and conv_ckpt [n][8192][3] instead, so a
// caller can commit any prefix of k accepted tokens by taking checkpoint k - 1 (bitwise what
// deltanet_seq_op would leave after those k tokens) and reject the rest by taking nothing.
template <int kBlock>
__device__ void deltanet_seq_ckpt_op(const DeltaNetSeqParams& p, float* state_ckpt,
                                     float* conv_ckpt, unsigned first, unsigned count) {
  dn_detail::seq_body<kBlock>(p, {nullptr, nullptr, state_ckpt, conv_ckpt}, first, count);
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) deltanet_seq_ckpt_kernel(DeltaNetSeqParams p,
                                                                   float* state_ckpt,
                                                                   float* conv_ckpt) {
  deltanet_seq_ckpt_op<kBlock>(p, state_ckpt, conv_ckpt, 0, deltanet_detail::kVHeads);
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) deltanet_seq_kernel(DeltaNetSeqParams p) {
  deltanet_seq_op<kBlock>(p, 0, deltanet_detail::kVHeads);
}

}  // namespace miso::kernels
