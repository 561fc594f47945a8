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
// thread, loaded and stored as 512-byte coalesced rows. deltanet_step_op (through
// dn_detail::token_update) and deltanet_seq_op (8 tokens per group: q / k / v, their norms, beta
// and decay formed for the group, then 2 barriers per token's state update) build every value from
// the same explicitly rounded helpers in the same order, so n steps and one n-token sequence agree
// bit for bit.

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

// The per-token arithmetic of the step and the sequence bodies. Every rounding is explicit (no
// multiply-add left for the compiler to contract or not), so both bodies give identical bits.
constexpr float kInvSqrtDim = 0.0883883476483184405501f;  // 1 / sqrt(128)

// 4-tap causal conv: taps 0..2 on the history (oldest first), tap 3 on the current input.
__device__ __forceinline__ float conv4(float w0, float w1, float w2, float w3, float h0, float h1,
                                       float h2, float x) {
  return __fmaf_rn(w3, x, __fmaf_rn(w2, h2, __fmaf_rn(w1, h1, __fmul_rn(w0, h0))));
}

__device__ __forceinline__ float beta_of(float b) { return 1.0f / (1.0f + __expf(-b)); }

__device__ __forceinline__ float decay_of(float a, float ssm_a, float dt_bias) {
  return __expf(__fmul_rn(ssm_a, softplus(__fadd_rn(a, dt_bias))));
}

// x / |x| given ss = the sum of squares of the vector.
__device__ __forceinline__ float l2_scale(float x, float ss) {
  return __fmul_rn(x, rsqrtf(__fadd_rn(ss, 1e-6f)));
}

// Gated RMSNorm of one output given ss = the sum of squares of the head's 128 outputs.
__device__ __forceinline__ float rms_gate(float o, float ss, float norm_w, float z, float eps) {
  const float r = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / kDim), eps));
  return __fmul_rn(__fmul_rn(__fmul_rn(o, r), norm_w), silu(z));
}

// Causal 4-tap conv of channel c for the current token, then SiLU; `own` also shifts the
// history of channel c into conv_out.
__device__ __forceinline__ float conv_step(const DeltaNetStepParams& p, unsigned c, bool own) {
  const float* hist = p.conv_in + 3 * c;
  const float* w = p.conv_w + 4 * c;
  const float x = p.qkv[c];
  const float y = conv4(w[0], w[1], w[2], w[3], hist[0], hist[1], hist[2], x);
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

// Decays the warp's 16 state rows (s[i] = row 16 w + i, columns 4 lane ..) and returns their part
// of S^T k; k16 = k[16 w ..].
__device__ __forceinline__ float4 decay_kv(float4 (&s)[16], const float* k16, float decay) {
  float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float kk = k16[i];
    s[i].x = __fmul_rn(s[i].x, decay), s[i].y = __fmul_rn(s[i].y, decay);
    s[i].z = __fmul_rn(s[i].z, decay), s[i].w = __fmul_rn(s[i].w, decay);
    kv.x = __fmaf_rn(s[i].x, kk, kv.x), kv.y = __fmaf_rn(s[i].y, kk, kv.y);
    kv.z = __fmaf_rn(s[i].z, kk, kv.z), kv.w = __fmaf_rn(s[i].w, kk, kv.w);
  }
  return kv;
}

// delta = beta (v - S^T k) for this lane's 4 columns from the 8 warps' partials (row stride 32
// float4), summed in warp order.
__device__ __forceinline__ float4 delta_of(const float4* part, float4 v4, float beta) {
  float4 acc = part[0];
#pragma unroll
  for (int r = 1; r < 8; ++r) {
    const float4 pr = part[32 * r];
    acc.x = __fadd_rn(acc.x, pr.x), acc.y = __fadd_rn(acc.y, pr.y);
    acc.z = __fadd_rn(acc.z, pr.z), acc.w = __fadd_rn(acc.w, pr.w);
  }
  return make_float4(__fmul_rn(__fsub_rn(v4.x, acc.x), beta), __fmul_rn(__fsub_rn(v4.y, acc.y), beta),
                     __fmul_rn(__fsub_rn(v4.z, acc.z), beta), __fmul_rn(__fsub_rn(v4.w, acc.w), beta));
}

// S += k delta^T on the warp's 16 rows; returns their part of S^T q.
__device__ __forceinline__ float4 update_o(float4 (&s)[16], const float* k16, const float* q16,
                                           float4 delta) {
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float kk = k16[i], qq = q16[i];
    s[i].x = __fmaf_rn(kk, delta.x, s[i].x), s[i].y = __fmaf_rn(kk, delta.y, s[i].y);
    s[i].z = __fmaf_rn(kk, delta.z, s[i].z), s[i].w = __fmaf_rn(kk, delta.w, s[i].w);
    o.x = __fmaf_rn(s[i].x, qq, o.x), o.y = __fmaf_rn(s[i].y, qq, o.y);
    o.z = __fmaf_rn(s[i].z, qq, o.z), o.w = __fmaf_rn(s[i].w, qq, o.w);
  }
  return o;
}

// Sum of the 8 warps' S^T q partials of column t, in warp order.
__device__ __forceinline__ float o_column(const float (&part)[8][kDim], unsigned t) {
  float oh = 0.0f;
#pragma unroll
  for (int r = 0; r < 8; ++r)
    oh = __fadd_rn(oh, part[r][t]);
  return oh;
}

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
  const float ss = wave_sum(__fmul_rn(x, x));
  if (lane == 0)
    sh.red[w] = ss;
  __syncthreads();
  if (t < kDim) {
    sh.q[t] = __fmul_rn(l2_scale(x, sh.red[0] + sh.red[1] + sh.red[2] + sh.red[3]), kInvSqrtDim);
  } else {
    sh.k[t - kDim] = l2_scale(x, sh.red[4] + sh.red[5] + sh.red[6] + sh.red[7]);
  }
  __syncthreads();
  const float beta = beta_of(beta_in);
  const float decay = decay_of(a_in, ssm_a, dt_bias);
  // Decay, then S^T k over this warp's 16 rows.
  reinterpret_cast<float4*>(sh.part[w])[lane] = decay_kv(s, sh.k + 16 * w, decay);
  __syncthreads();
  const float4 delta = delta_of(reinterpret_cast<const float4*>(sh.part[0]) + lane,
                                reinterpret_cast<const float4*>(sh.v)[lane], beta);
  __syncthreads();  // everyone has read part[] before it is reused
  reinterpret_cast<float4*>(sh.part[w])[lane] = update_o(s, sh.k + 16 * w, sh.q + 16 * w, delta);
  __syncthreads();
  // Gated RMSNorm over the 128 outputs (warps 0-3, one column per thread).
  const float oh = t < kDim ? o_column(sh.part, t) : 0.0f;
  const float os = wave_sum(__fmul_rn(oh, oh));
  __syncthreads();  // part[] / red[] reads done before red[] is rewritten
  if (lane == 0 && w < 4)
    sh.red[w] = os;
  __syncthreads();
  if (t < kDim)
    out[t] = rms_gate(oh, sh.red[0] + sh.red[1] + sh.red[2] + sh.red[3], norm_w_t, z_t, eps);
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

// Tokens per group of the sequence body. A token's q / k / v, their L2 norms, beta and decay do
// not depend on the state, so they are formed for a whole group at once (2 barriers); the state
// update then takes 2 barriers per token and the gated norms of the group 1 more (7 per token when
// every token runs token_update). The float operations and their order are those of
// token_update, so a sequence still agrees bit for bit with n single steps.
constexpr unsigned kSeqGroup = 8;

struct SeqShared {
  float q[kSeqGroup][kDim], k[kSeqGroup][kDim], v[kSeqGroup][kDim];
  float part[2][8][kDim];  // [0]: S^T k partials of the 8 warps, [1]: S^T q partials
  float red[kSeqGroup][8];   // q / k sums of squares per warp
  float red2[kSeqGroup][4];  // output sums of squares per warp
};

template <int kBlock>
__device__ void seq_body(const DeltaNetSeqParams& p, const SeqSinks& out, unsigned first,
                         unsigned count) {
  using namespace deltanet_detail;
  static_assert(kBlock == 2 * kDim, "eight warps of 16 state rows each");
  constexpr unsigned G = kSeqGroup;
  constexpr unsigned kOut = kVHeads * kDim;
  constexpr std::size_t kStateFloats = std::size_t{kVHeads} * kDim * kDim;
  constexpr std::size_t kConvFloats = std::size_t{3} * (2 * kKHeads + kVHeads) * kDim;
  __shared__ SeqShared sh;
  const unsigned t = threadIdx.x, w = t / 32, lane = t % 32;
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
    load_state(s, S);
    const float nw = t < kDim ? p.norm_w[t] : 0.0f;
    const float ssm_a_h = p.ssm_a[h], dt_bias_h = p.dt_bias[h];
    // The raw inputs of a group (conv inputs x0 / x1, b, a and the gate z[t]) are loaded one
    // group ahead, so their memory latency overlaps the previous group's updates.
    float nx0[G], nx1[G], nb[G], na[G], nz[G];
    auto load_group = [&](unsigned g0) {
#pragma unroll
      for (unsigned j = 0; j < G; ++j) {
        nx0[j] = nx1[j] = nb[j] = na[j] = nz[j] = 0.0f;
        if (g0 + j < p.n) {
          const float* x = p.qkv + std::size_t{g0 + j} * p.qkv_stride;
          const std::size_t zrow = std::size_t{g0 + j} * p.zab_stride;
          nx0[j] = x[c0];
          if (t < kDim) {
            nx1[j] = x[c1];
            nz[j] = p.z[zrow + h * kDim + t];
          }
          nb[j] = p.b[zrow + h];
          na[j] = p.a[zrow + h];
        }
      }
    };
    if (p.n > 0)
      load_group(0);
    for (unsigned g0 = 0; g0 < p.n; g0 += G) {
      const unsigned gcount = p.n - g0 < G ? p.n - g0 : G;
      float x0[G], x1[G], bj[G], aj[G], zj[G];
#pragma unroll
      for (unsigned j = 0; j < G; ++j)
        x0[j] = nx0[j], x1[j] = nx1[j], bj[j] = nb[j], aj[j] = na[j], zj[j] = nz[j];
      if (g0 + G < p.n)
        load_group(g0 + G);
      // Conv + SiLU of the group's tokens (each thread its own channels, in token order), and
      // the per-warp sums of squares of q / k.
      float y[G];
#pragma unroll
      for (unsigned j = 0; j < G; ++j) {
        if (j < gcount) {
          const float y0 = silu(conv4(w0[0], w0[1], w0[2], w0[3], h0[0], h0[1], h0[2], x0[j]));
          h0[0] = h0[1], h0[1] = h0[2], h0[2] = x0[j];
          if (t < kDim) {
            const float y1 = silu(conv4(w1[0], w1[1], w1[2], w1[3], h1[0], h1[1], h1[2], x1[j]));
            h1[0] = h1[1], h1[1] = h1[2], h1[2] = x1[j];
            sh.v[j][t] = y1;
          }
          y[j] = y0;
          const float ss = wave_sum(__fmul_rn(y0, y0));
          if (lane == 0)
            sh.red[j][w] = ss;
          if (out.conv_ckpt != nullptr) {
            float* cc = out.conv_ckpt + (g0 + j) * kConvFloats;
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
      }
      __syncthreads();
#pragma unroll
      for (unsigned j = 0; j < G; ++j) {
        if (j < gcount) {
          if (t < kDim) {
            sh.q[j][t] = __fmul_rn(
                l2_scale(y[j], sh.red[j][0] + sh.red[j][1] + sh.red[j][2] + sh.red[j][3]),
                kInvSqrtDim);
          } else {
            sh.k[j][t - kDim] =
                l2_scale(y[j], sh.red[j][4] + sh.red[j][5] + sh.red[j][6] + sh.red[j][7]);
          }
        }
      }
      __syncthreads();
      // The delta rule, token by token.
      float oh[G];
#pragma unroll
      for (unsigned j = 0; j < G; ++j) {
        oh[j] = 0.0f;
        if (j < gcount) {
          const float beta = beta_of(bj[j]);
          const float decay = decay_of(aj[j], ssm_a_h, dt_bias_h);
          reinterpret_cast<float4*>(sh.part[0][w])[lane] = decay_kv(s, sh.k[j] + 16 * w, decay);
          __syncthreads();
          const float4 delta = delta_of(reinterpret_cast<const float4*>(sh.part[0][0]) + lane,
                                        reinterpret_cast<const float4*>(sh.v[j])[lane], beta);
          // part[1] was last read (previous token) before this token's barrier above, part[0]
          // is read by every thread before it reaches the barrier below.
          reinterpret_cast<float4*>(sh.part[1][w])[lane] =
              update_o(s, sh.k[j] + 16 * w, sh.q[j] + 16 * w, delta);
          __syncthreads();
          if (t < kDim)
            oh[j] = o_column(sh.part[1], t);
          if (out.state_ckpt != nullptr)
            store_state(s, out.state_ckpt + (g0 + j) * kStateFloats + std::size_t{h} * kDim * kDim);
        }
      }
      // Gated RMSNorm of the group's outputs (warps 0-3, one column per thread).
#pragma unroll
      for (unsigned j = 0; j < G; ++j) {
        if (j < gcount && w < 4) {
          const float os = wave_sum(__fmul_rn(oh[j], oh[j]));
          if (lane == 0)
            sh.red2[j][w] = os;
        }
      }
      __syncthreads();
#pragma unroll
      for (unsigned j = 0; j < G; ++j) {
        if (j < gcount && t < kDim) {
          p.out[std::size_t{g0 + j} * kOut + h * kDim + t] = rms_gate(
              oh[j], sh.red2[j][0] + sh.red2[j][1] + sh.red2[j][2] + sh.red2[j][3], nw, zj[j],
              p.eps);
        }
      }
    }
    if (out.state != nullptr)
      store_state(s, out.state + std::size_t{h} * kDim * kDim);
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
