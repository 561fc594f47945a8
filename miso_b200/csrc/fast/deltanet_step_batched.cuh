#pragma once

// Batched Gated DeltaNet decode step: the per-token arithmetic of deltanet_step_op
// (kernels/deltanet_step.hpp) for `batch` independent sequences in one launch, the fast path
// behind miso_deltanet_step_batched().
//
// The step reads and writes every sequence's 32 x 128 x 128 fp32 state once (128 KB per
// (sequence, head) of traffic, 268 MB per step at batch 64), so it is HBM-bound. A persistent
// kernel, two 512-thread CTAs per SM, walks the (sequence, head) units: each unit's 64 KB state
// arrives by a bulk copy into shared memory, goes to registers (warp w: state rows (k)
// [8w, 8w + 8), lane l: value columns [4l, 4l + 4)) and, updated, straight back to global
// memory; as soon as a state is in registers the copy of the CTA's next unit starts, so it lands
// while this one is computed, and the two CTAs of an SM overlap each other's compute phases. The
// next unit's conv inputs, betas, decays and gate are loaded into registers likewise.

#include <cuda_runtime.h>

#include <cstdint>

#include "../common/device.cuh"
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

constexpr int kStages = 1;
constexpr int kCtasPerSm = 2;
constexpr uint32_t kStateBytes = kDim * kDim * 4;  // 64 KB
constexpr size_t kSmemBytes = kStages * size_t(kStateBytes) + 64;

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ float conv1(const float* w, const float* hist, float x) {
  return silu(w[0] * hist[0] + w[1] * hist[1] + w[2] * hist[2] + w[3] * x);
}

// The per-unit inputs other than the state, gathered ahead of their use.
struct UnitIn {
  float x, h0, h1, h2, w0, w1, w2, w3;  // conv inputs of the thread's channel (t < 384)
  float a, b, z;                        // the unit's a, b and the thread's gate (t < 128)
};

__device__ __forceinline__ void load_unit(const Args& p, unsigned u, unsigned t, UnitIn& in) {
  const unsigned bq = u / kVHeads, h = u % kVHeads, kh = h % kKHeads;
  if (t < 3 * kDim) {
    const unsigned which = t / kDim, i = t % kDim;
    const unsigned c = which == 0 ? kh * kDim + i
                     : which == 1 ? kKHeads * kDim + kh * kDim + i
                                  : 2 * kKHeads * kDim + h * kDim + i;
    const float* hist = p.conv_in + size_t(bq) * kCh * 3 + 3 * c;
    in.x = p.qkv[size_t(bq) * p.in_stride + c];
    in.h0 = hist[0], in.h1 = hist[1], in.h2 = hist[2];
    const float4 w = *reinterpret_cast<const float4*>(p.conv_w + 4 * c);
    in.w0 = w.x, in.w1 = w.y, in.w2 = w.z, in.w3 = w.w;
  }
  in.a = p.a[size_t(bq) * p.in_stride + h];
  in.b = p.b[size_t(bq) * p.in_stride + h];
  in.z = t < kDim ? p.z[size_t(bq) * p.in_stride + h * kDim + t] : 0.0f;
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm) step_batched_kernel(Args p) {
  using miso::kernels::wave_sum;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float qs[kDim], ks[kDim], vs[kDim];
  __shared__ float part[kWarps][kDim];
  __shared__ float red[kWarps];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * size_t(kStateBytes));
  const unsigned t = threadIdx.x, w = t / 32, lane = t % 32;
  const unsigned units = p.batch * kVHeads, G = gridDim.x;
  if (t == 0) {
    for (int i = 0; i < kStages; ++i)
      dev::mbar_init(dev::smem_u32(&full[i]), 1);
    dev::mbar_init_fence();
  }
  __syncthreads();
  auto issue = [&](unsigned i) {  // local unit i -> stage i % kStages
    const unsigned u = blockIdx.x + i * G;
    const uint32_t bar = dev::smem_u32(&full[i % kStages]);
    dev::mbar_arrive_expect_tx(bar, kStateBytes);
    dev::bulk_load(dev::smem_u32(smem + (i % kStages) * size_t(kStateBytes)),
                   p.state + size_t(u) * kDim * kDim, kStateBytes, bar);
  };
  const unsigned n_local = blockIdx.x < units ? (units - blockIdx.x + G - 1) / G : 0;
  if (t == 0)
    for (unsigned i = 0; i < kStages && i < n_local; ++i)
      issue(i);
  UnitIn in{}, nxt{};
  if (n_local > 0)
    load_unit(p, blockIdx.x, t, in);

  for (unsigned i = 0; i < n_local; ++i) {
    const unsigned u = blockIdx.x + i * G, bq = u / kVHeads, h = u % kVHeads;
    const unsigned kh = h % kKHeads;
    const bool own_qk = h < kKHeads;
    if (!dev::mbar_wait(dev::smem_u32(&full[i % kStages]), (i / kStages) & 1, 0x14))
      break;  // (a timed-out unit leaves its state unchanged; the status word says so)
    const float4* Ssm = reinterpret_cast<const float4*>(smem + (i % kStages) * size_t(kStateBytes)) +
                        (kRowsPerWarp * w) * (kDim / 4) + lane;
    float4 s[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
      s[r] = Ssm[r * (kDim / 4)];
    dev::fence_proxy_async_smem();
    __syncthreads();  // the stage has been read: refill it with the unit kStages ahead
    if (t == 0 && i + kStages < n_local)
      issue(i + kStages);
    float4* S = reinterpret_cast<float4*>(p.state + size_t(u) * kDim * kDim) +
                (kRowsPerWarp * w) * (kDim / 4) + lane;
    float* cout = p.conv_out + size_t(bq) * kCh * 3;

    // Conv + SiLU of this head's 384 channels: threads [0,128) q, [128,256) k, [256,384) v.
    if (t < 3 * kDim) {
      const unsigned which = t / kDim, ii = t % kDim;
      const unsigned c = which == 0 ? kh * kDim + ii
                       : which == 1 ? kKHeads * kDim + kh * kDim + ii
                                    : 2 * kKHeads * kDim + h * kDim + ii;
      const float cw[4] = {in.w0, in.w1, in.w2, in.w3}, hist[3] = {in.h0, in.h1, in.h2};
      const float y = conv1(cw, hist, in.x);
      if (which == 2 || own_qk) {
        cout[3 * c] = in.h1;
        cout[3 * c + 1] = in.h2;
        cout[3 * c + 2] = in.x;
      }
      (which == 0 ? qs : which == 1 ? ks : vs)[ii] = y;
    }
    // The rest of this unit needs only these three of its inputs: load the next unit's now.
    const float beta = 1.0f / (1.0f + __expf(-in.b));
    const float decay = __expf(p.ssm_a[h] * miso::kernels::deltanet_detail::softplus(
                                                in.a + p.dt_bias[h]));
    const float gz = silu(in.z);
    if (i + 1 < n_local)
      load_unit(p, u + G, t, nxt);
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
    float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const float kk = ks[kRowsPerWarp * w + r];
      s[r].x *= decay, s[r].y *= decay, s[r].z *= decay, s[r].w *= decay;
      kv.x += s[r].x * kk, kv.y += s[r].y * kk, kv.z += s[r].z * kk, kv.w += s[r].w * kk;
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
    for (int r = 0; r < kRowsPerWarp; ++r) {
      const float kk = ks[kRowsPerWarp * w + r], qq = qs[kRowsPerWarp * w + r];
      s[r].x += kk * delta.x, s[r].y += kk * delta.y, s[r].z += kk * delta.z,
          s[r].w += kk * delta.w;
      o.x += s[r].x * qq, o.y += s[r].y * qq, o.z += s[r].z * qq, o.w += s[r].w * qq;
      S[r * (kDim / 4)] = s[r];
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
      const float rr = rsqrtf((red[0] + red[1] + red[2] + red[3]) / kDim + p.eps);
      p.out[size_t(bq) * kVHeads * kDim + h * kDim + t] = oh * rr * p.norm_w[t] * gz;
    }
    __syncthreads();  // qs / ks / vs / part / red free for the next unit
    in = nxt;
  }
  // No thread leaves while a bulk copy into this CTA's shared memory may still be landing
  // (after a timed-out wait): wait (bounded) for every issued stage.
  if (t == 0)
    for (unsigned i = 0; i < kStages && i < n_local; ++i) {
      const unsigned last = n_local - 1 - i;  // the copies of the last kStages units
      dev::mbar_wait(dev::smem_u32(&full[last % kStages]), (last / kStages) & 1);
    }
  __syncthreads();
}

}  // namespace miso::fast::dnstep
