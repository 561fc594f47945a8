#pragma once

// Batched Gated DeltaNet decode step: the per-token arithmetic of deltanet_step_op
// (kernels/deltanet_step.hpp) for `batch` independent sequences in one launch, the fast path
// behind miso_deltanet_step_batched().
//
// The step reads and writes every sequence's 32 x 128 x 128 fp32 state once (128 KB per
// (sequence, head) of traffic, 268 MB per step at batch 64), so it is HBM-bound. One 512-thread
// block per (V head, sequence): warp w holds state rows (k index) [8w, 8w + 8) and lane l value
// columns [4l, 4l + 4) — 8 float4 registers per thread, loaded as 512-byte coalesced rows, all
// issued before the first use — and two blocks fit on an SM (64 registers a thread), so 128 KB
// of state loads are in flight per SM.

#include <cuda_runtime.h>

#include <cstdint>

#include "../kernels/deltanet_step.hpp"

namespace miso::fast::dnstep {

constexpr int kDim = 128, kKHeads = 16, kVHeads = 32, kCh = 8192;
constexpr int kWarps = 16, kThreads = kWarps * 32, kRowsPerWarp = kDim / kWarps;

struct Args {
  const float* qkv;
  const float* z;
  const float* a;
  const float* b;
  const float* conv_w;
  const float* ssm_a;
  const float* dt_bias;
  const float* norm_w;
  const float* conv_in;
  float* conv_out;
  float* state;
  float* out;
  unsigned batch, in_stride;
  float eps;
};

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ float conv1(const float* w, const float* hist, float x) {
  return silu(w[0] * hist[0] + w[1] * hist[1] + w[2] * hist[2] + w[3] * x);
}

__global__ void __launch_bounds__(kThreads, 2) step_batched_kernel(Args p) {
  using miso::kernels::wave_sum;
  __shared__ float qs[kDim], ks[kDim], vs[kDim];
  __shared__ float part[kWarps][kDim];
  __shared__ float red[kWarps];
  const unsigned h = blockIdx.x, bq = blockIdx.y;
  const unsigned t = threadIdx.x, w = t / 32, lane = t % 32;
  const unsigned kh = h % kKHeads;
  const bool own_qk = h < kKHeads;
  const float* x = p.qkv + size_t(bq) * p.in_stride;
  const float* cin = p.conv_in + size_t(bq) * kCh * 3;
  float* cout = p.conv_out + size_t(bq) * kCh * 3;
  float4* S = reinterpret_cast<float4*>(p.state + (size_t(bq) * kVHeads + h) * kDim * kDim) +
              (kRowsPerWarp * w) * (kDim / 4) + lane;

  float4 s[kRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
    s[i] = S[i * (kDim / 4)];

  // Conv + SiLU of this head's 384 channels: threads [0,128) q, [128,256) k, [256,384) v.
  if (t < 3 * kDim) {
    const unsigned which = t / kDim, i = t % kDim;
    const unsigned c = which == 0 ? kh * kDim + i
                     : which == 1 ? kKHeads * kDim + kh * kDim + i
                                  : 2 * kKHeads * kDim + h * kDim + i;
    const float* hist = cin + 3 * c;
    const float xc = x[c];
    const float y = conv1(p.conv_w + 4 * c, hist, xc);
    if (which == 2 || own_qk) {
      cout[3 * c] = hist[1];
      cout[3 * c + 1] = hist[2];
      cout[3 * c + 2] = xc;
    }
    (which == 0 ? qs : which == 1 ? ks : vs)[i] = y;
  }
  __syncthreads();
  // L2 norms: warps 0-3 reduce q, warps 4-7 reduce k.
  if (w < 8) {
    const float xv = w < 4 ? qs[t] : ks[t - kDim];
    const float ss = wave_sum(xv * xv);
    if (lane == 0)
      red[w] = ss;
  }
  __syncthreads();
  if (t < kDim) {
    qs[t] = qs[t] * rsqrtf(red[0] + red[1] + red[2] + red[3] + 1e-6f) *
            rsqrtf(static_cast<float>(kDim));
  } else if (t < 2 * kDim) {
    ks[t - kDim] = ks[t - kDim] * rsqrtf(red[4] + red[5] + red[6] + red[7] + 1e-6f);
  }
  __syncthreads();
  const float* zb = p.z + size_t(bq) * p.in_stride;
  const float beta = 1.0f / (1.0f + __expf(-p.b[size_t(bq) * p.in_stride + h]));
  const float decay =
      __expf(p.ssm_a[h] * miso::kernels::deltanet_detail::softplus(
                              p.a[size_t(bq) * p.in_stride + h] + p.dt_bias[h]));
  float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const float kk = ks[kRowsPerWarp * w + i];
    s[i].x *= decay, s[i].y *= decay, s[i].z *= decay, s[i].w *= decay;
    kv.x += s[i].x * kk, kv.y += s[i].y * kk, kv.z += s[i].z * kk, kv.w += s[i].w * kk;
  }
  reinterpret_cast<float4*>(part[w])[lane] = kv;
  __syncthreads();
  float4 delta;
  {
    float4 acc = reinterpret_cast<const float4*>(part[0])[lane];
#pragma unroll
    for (int r = 1; r < kWarps; ++r) {
      const float4 pr = reinterpret_cast<const float4*>(part[r])[lane];
      acc.x += pr.x, acc.y += pr.y, acc.z += pr.z, acc.w += pr.w;
    }
    const float4 v4 = reinterpret_cast<const float4*>(vs)[lane];
    delta = make_float4((v4.x - acc.x) * beta, (v4.y - acc.y) * beta, (v4.z - acc.z) * beta,
                        (v4.w - acc.w) * beta);
  }
  __syncthreads();
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const float kk = ks[kRowsPerWarp * w + i], qq = qs[kRowsPerWarp * w + i];
    s[i].x += kk * delta.x, s[i].y += kk * delta.y, s[i].z += kk * delta.z, s[i].w += kk * delta.w;
    o.x += s[i].x * qq, o.y += s[i].y * qq, o.z += s[i].z * qq, o.w += s[i].w * qq;
    S[i * (kDim / 4)] = s[i];
  }
  reinterpret_cast<float4*>(part[w])[lane] = o;
  __syncthreads();
  // Gated RMSNorm over the 128 outputs (warps 0-3, one column per thread).
  float oh = 0.0f;
  if (t < kDim) {
#pragma unroll
    for (int r = 0; r < kWarps; ++r)
      oh += part[r][t];
  }
  const float os = wave_sum(oh * oh);
  __syncthreads();
  if (lane == 0 && w < 4)
    red[w] = os;
  __syncthreads();
  if (t < kDim) {
    const float r = rsqrtf((red[0] + red[1] + red[2] + red[3]) / kDim + p.eps);
    p.out[size_t(bq) * kVHeads * kDim + h * kDim + t] =
        oh * r * p.norm_w[t] * silu(zb[h * kDim + t]);
  }
}

}  // namespace miso::fast::dnstep
