#pragma once

// Gated DeltaNet prefill (chunked gated delta rule, chunk 64) on the 5th-generation tensor cores:
// the fast path behind miso_deltanet_prefill_tc(). Same inputs, outputs and conv / state
// conventions as the n-token recurrence deltanet_seq (reference kernels/deltanet_step.hpp:146-273
// and kernels/deltanet_chunk.hpp:3-9 for the chunk algebra).
//
// Per V head h (K head kh = h % 16) and chunk of C = 64 tokens with in-chunk cumulative log decay
// g_i = sum_{t <= i} log(alpha_t), the chunk update of the state S [k][v] is
//   L    = strictly_lower(beta_i e^(g_i - g_j) k_i . k_j),   T = (I + L)^-1   (UT transform)
//   W    = T diag(beta e^g) K,   U = T diag(beta) V                           (WY form)
//   delta = U - W S                                    (the delta-rule corrections of the chunk)
//   O    = diag(e^g) Q S + Aqk delta,  Aqk = lower_incl(e^(g_i - g_j) q_i . k_j)
//   S   <- e^(g_last) S + K^T diag(e^(g_last - g)) delta
// and out = O * rsqrt(mean(O^2) + eps) * norm_w * SiLU(z) per token and head.
//
// Three launches:
//   conv_kernel     one block per (1024 channels, 16 tokens): 4-tap causal conv + SiLU, q / k
//                   L2 norms (q also * 1/sqrt(128)), beta, log alpha; writes q, k, v as fp16
//                   and the final conv history.
//   prepare_kernel  one block per (chunk, K head), both V heads of the K head: [K; Q] K^T as one
//                   tcgen05 MMA (M=128, N=64, K=128), L and Aqk from it, T = (I + L)^-1 by
//                   forward substitution (thread per column), Tw = T diag(beta e^g),
//                   Tu = T diag(beta) and Aqk as fp16 tiles, e^g and e^(g_last - g) as fp32.
//   recur_kernel    one block per V head, the 128 x 128 state transposed (S^T: lane = v, column =
//                   k) as an fp32 TMEM accumulator; per chunk five tcgen05 MMA groups with M = 128:
//                     W^T = K^T Tw^T, U^T = V^T Tu^T    (from this chunk's inputs only)
//                     X^T = S^T W^T,  Y^T = S^T Q^T     (A = S^T as fp16 in shared memory)
//                     S^T += (delta^T diag(e^(g_last - g))) K
//                     Z^T = delta^T Aqk^T
//                   and the epilogues delta^T = U^T - X^T, O^T = diag(e^g) Y^T + Z^T (+ norm,
//                   gate, store) on CUDA cores.
//
// Precision: every MMA accumulates in fp32 and the state stays fp32 in TMEM; the operands (q, k,
// v, T, Aqk, the fp16 copy of S^T read by X / Y, delta) are fp16, whose 11-bit significand keeps
// the outputs within ~1e-4 relative of an fp64 recurrence.
//
// Every mbarrier wait is bounded; on a timeout the block records MISO_STATUS_TIMEOUT (site 0x30 /
// 0x31), stops issuing, drains what it issued and frees its TMEM before exiting.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../common/device.cuh"
#include "../common/tcgen05.cuh"

namespace miso::fast::dnchunk {

constexpr int kKHeads = 16, kVHeads = 32, kDim = 128, kC = 64;
constexpr int kQkCh = kKHeads * kDim;              // 2048 q (or k) channels
constexpr int kCh = 2 * kQkCh + kVHeads * kDim;    // 8192 conv channels
constexpr uint32_t kTile = kC * 64 * 2;            // one [64 rows][64] fp16 box: 8 KB

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }
// SiLU with the fast (2 ulp) division; well inside the fp16-operand error of this path.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(__expf(x)); }

__device__ __forceinline__ uint32_t h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Two-term fp16 split of four fp32 values: x = hi + lo with both fp16, so that products of split
// operands (hi * hi + hi * lo + lo * hi) keep close to fp32 accuracy.
__device__ __forceinline__ void split4(const float (&y)[4], uint2& hi, uint2& lo) {
  const __half2 a = __floats2half2_rn(y[0], y[1]), b = __floats2half2_rn(y[2], y[3]);
  const float2 fa = __half22float2(a), fb = __half22float2(b);
  hi = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  lo = make_uint2(h2(y[0] - fa.x, y[1] - fa.y), h2(y[2] - fb.x, y[3] - fb.y));
}

// ================================================================================ conv_kernel

struct ConvArgs {
  const float* qkv;  // [n][qkv_stride]: q 2048 | k 2048 | v 4096
  const float* a;    // a[t * zab_stride + h]
  const float* b;
  const float* conv_w;   // [8192][4]
  const float* conv_in;  // [8192][3] oldest first
  float* conv_out;
  const float* ssm_a;
  const float* dt_bias;
  __half* q16;    // [n][16][128] fp16 value (high part)
  __half* k16;    // [n][16][128]
  __half* v16;    // [n][32][128]
  __half* q16lo;  // fp16 remainders x - hi, same layouts
  __half* k16lo;
  __half* v16lo;
  float* beta;  // [32][np]
  float* loga;  // [32][np]
  unsigned n, np, qkv_stride, zab_stride;
};

constexpr int kConvThreads = 256;
constexpr int kConvTokens = 16;  // tokens per block: the block's conv weights are read once

// Block (m, y): channels [1024 m, 1024 m + 1024) of tokens [16 y, 16 y + 16). Thread t owns the
// four channels 1024 m + 4 t .. + 3, so a warp covers one whole 128-channel head (m = 0, 1: q
// heads; 2, 3: k heads; 4..7: v heads) and the q / k L2 norms are warp reductions. The 4-tap
// window slides along the block's tokens in registers.
__global__ void __launch_bounds__(kConvThreads) conv_kernel(ConvArgs a) {
  const unsigned m = blockIdx.x, t0 = blockIdx.y * kConvTokens, tid = threadIdx.x,
                 lane = tid % 32, warp = tid / 32;
  const unsigned c = 1024 * m + 4 * tid;
  const float4* w4 = reinterpret_cast<const float4*>(a.conv_w + 4 * size_t(c));
  const float4 w0 = w4[0], w1 = w4[1], w2 = w4[2], w3 = w4[3];
  float4 h[3];  // x_{t-3}, x_{t-2}, x_{t-1} of the current token
#pragma unroll
  for (int s = 0; s < 3; ++s) {
    const int tt = int(t0) - 3 + s;
    if (tt >= 0) {
      h[s] = *reinterpret_cast<const float4*>(a.qkv + size_t(tt) * a.qkv_stride + c);
    } else {
      const int slot = tt + 3;
      h[s] = make_float4(a.conv_in[3 * c + slot], a.conv_in[3 * (c + 1) + slot],
                         a.conv_in[3 * (c + 2) + slot], a.conv_in[3 * (c + 3) + slot]);
    }
  }
  float4 xs[kConvTokens];
#pragma unroll
  for (int i = 0; i < kConvTokens; ++i)
    xs[i] = t0 + i < a.n
                ? *reinterpret_cast<const float4*>(a.qkv + size_t(t0 + i) * a.qkv_stride + c)
                : make_float4(0.f, 0.f, 0.f, 0.f);
  if (t0 == 0 && a.n < 3) {  // history slots older than the sequence come from conv_in
    for (unsigned slot = 0; slot + a.n < 3; ++slot)
      for (int e = 0; e < 4; ++e)
        a.conv_out[3 * (c + e) + slot] = a.conv_in[3 * (c + e) + slot + a.n];
  }
#pragma unroll
  for (int i = 0; i < kConvTokens; ++i) {
    const unsigned t = t0 + i;
    if (t >= a.n)
      break;
    const float4 x = xs[i];
    float y[4];
    y[0] = silu_fast(w0.x * h[0].x + w0.y * h[1].x + w0.z * h[2].x + w0.w * x.x);
    y[1] = silu_fast(w1.x * h[0].y + w1.y * h[1].y + w1.z * h[2].y + w1.w * x.y);
    y[2] = silu_fast(w2.x * h[0].z + w2.y * h[1].z + w2.z * h[2].z + w2.w * x.z);
    y[3] = silu_fast(w3.x * h[0].w + w3.y * h[1].w + w3.z * h[2].w + w3.w * x.w);
    h[0] = h[1], h[1] = h[2], h[2] = x;
    if (t + 3 >= a.n) {  // the last three inputs become the conv history
      const unsigned slot = t + 3 - a.n;
      a.conv_out[3 * c + slot] = x.x;
      a.conv_out[3 * (c + 1) + slot] = x.y;
      a.conv_out[3 * (c + 2) + slot] = x.z;
      a.conv_out[3 * (c + 3) + slot] = x.w;
    }
    if (m < 4) {
      float ss = y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
        ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float r = rsqrtf(ss + 1e-6f);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        y[e] *= r;
      if (m < 2) {
        const float qs = rsqrtf(static_cast<float>(kDim));
#pragma unroll
        for (int e = 0; e < 4; ++e)
          y[e] *= qs;
      }
      const unsigned head = (c % kQkCh) / kDim;
      const size_t off = (size_t(t) * kKHeads + head) * kDim + c % kDim;
      uint2 hi, lo;
      split4(y, hi, lo);
      *reinterpret_cast<uint2*>((m < 2 ? a.q16 : a.k16) + off) = hi;
      *reinterpret_cast<uint2*>((m < 2 ? a.q16lo : a.k16lo) + off) = lo;
    } else {
      const size_t off = size_t(t) * kVHeads * kDim + (c - 2 * kQkCh);
      uint2 hi, lo;
      split4(y, hi, lo);
      *reinterpret_cast<uint2*>(a.v16 + off) = hi;
      *reinterpret_cast<uint2*>(a.v16lo + off) = lo;
    }
  }
  if (m == 0 && warp == 0) {
    for (unsigned i = 0; i < kConvTokens && t0 + i < a.n; ++i) {
      const unsigned t = t0 + i, hh = lane;
      const float bv = a.b[size_t(t) * a.zab_stride + hh];
      const float av = a.a[size_t(t) * a.zab_stride + hh];
      a.beta[size_t(hh) * a.np + t] = 1.0f / (1.0f + __expf(-bv));
      a.loga[size_t(hh) * a.np + t] = a.ssm_a[hh] * softplus(av + a.dt_bias[hh]);
    }
  }
}

// ============================================================================= prepare_kernel

struct PrepareArgs {
  const float* beta;  // [32][np]
  const float* loga;  // [32][np]
  float* eg;          // [32][np] e^(g_t), g = in-chunk cumulative log decay (0 past n)
  float* egl;         // [32][np] e^(g_last - g_t), g_last that of the chunk's row 63
  __half* tw;         // [32][nc][64][64]
  __half* tu;
  __half* aqk;        // Aqk as fp16 high part ...
  __half* aqklo;      // ... and fp16 remainder
  unsigned n, np, nc;
};

constexpr int kPrepThreads = 128;
constexpr int kLRow = 68;  // fp32 row stride of L (16-byte aligned rows)
constexpr int kTRow = 65;  // fp32 stride of a solved column of T (conflict-free per lane)
static_assert((2 * 64 * kTRow + 4 * 64) * 4 <= 8 * 8192, "T columns fit in the [K; Q] tile area");
// [K; Q] as fp16 high parts (32 KB) then remainders (32 KB): 64-dim slab s of part p at
// 32 KB p + 16 KB s, K rows first, Q rows 8 KB later (M = 128 rows).
constexpr uint32_t kPrepOffL = 8 * kTile;
constexpr uint32_t kPrepOffG = kPrepOffL + 2 * kC * kLRow * 4;     // g[2][64], beta[2][64]
constexpr uint32_t kPrepOffBar = kPrepOffG + 4 * kC * 4;
constexpr size_t kPrepSmemBytes = kPrepOffBar + 64;

__global__ void __launch_bounds__(kPrepThreads, 2)
    prepare_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap qlmap,
                   const __grid_constant__ CUtensorMap klmap, PrepareArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((dev::smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0)
      dev::set_status(dev::kStatusTimeout, 0x31);
    return;
  }
  const unsigned c = blockIdx.x, kh = blockIdx.y, tid = threadIdx.x, warp = tid / 32,
                 lane = tid % 32;
  const uint32_t sbase = dev::smem_u32(smem);
  float* Ls = reinterpret_cast<float*>(smem + kPrepOffL);  // [2][64][kLRow]
  float* gs = reinterpret_cast<float*>(smem + kPrepOffG);  // [2][64]
  float* bs = gs + 2 * kC;                                 // [2][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPrepOffBar);  // load, mma
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  int* fail = reinterpret_cast<int*>(bars + 3);

  if (tid == 0) {
    dev::mbar_init(dev::smem_u32(&bars[0]), 1);
    dev::mbar_init(dev::smem_u32(&bars[1]), 1);
    *fail = 0;
    dev::mbar_init_fence();
  }
  if (warp == 0) {
    dev::tmem_alloc(dev::smem_u32(tmem_slot), 64);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {
    dev::mbar_arrive_expect_tx(dev::smem_u32(&bars[0]), 8 * kTile);
    for (int part = 0; part < 2; ++part)
      for (int sl = 0; sl < 2; ++sl) {
        const uint32_t dst = sbase + part * 4 * kTile + sl * 2 * kTile;
        dev::tma_load_3d(dst, part ? &klmap : &kmap, sl * 64, kh, c * kC, dev::smem_u32(&bars[0]));
        dev::tma_load_3d(dst + kTile, part ? &qlmap : &qmap, sl * 64, kh, c * kC,
                         dev::smem_u32(&bars[0]));
      }
  }
  if (warp < 2) {
    // In-chunk cumulative log decay and beta of V head kh + 16 warp (zero past n).
    const unsigned h = kh + kKHeads * warp;
    const unsigned t0 = c * kC + 2 * lane;
    const float l0 = t0 < a.n ? a.loga[size_t(h) * a.np + t0] : 0.0f;
    const float l1 = t0 + 1 < a.n ? a.loga[size_t(h) * a.np + t0 + 1] : 0.0f;
    float incl = l0 + l1;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= unsigned(off))
        incl += y;
    }
    const float g0 = incl - l1, g1 = incl;
    const float glast = __shfl_sync(0xffffffffu, incl, 31);
    gs[warp * kC + 2 * lane] = g0;
    gs[warp * kC + 2 * lane + 1] = g1;
    bs[warp * kC + 2 * lane] = t0 < a.n ? a.beta[size_t(h) * a.np + t0] : 0.0f;
    bs[warp * kC + 2 * lane + 1] = t0 + 1 < a.n ? a.beta[size_t(h) * a.np + t0 + 1] : 0.0f;
    *reinterpret_cast<float2*>(a.eg + size_t(h) * a.np + t0) =
        make_float2(__expf(g0), __expf(g1));
    *reinterpret_cast<float2*>(a.egl + size_t(h) * a.np + t0) =
        make_float2(__expf(glast - g0), __expf(glast - g1));
  }
  if (tid == 0) {
    if (dev::mbar_wait(dev::smem_u32(&bars[0]), 0, 0x31)) {
      dev::tc_fence_after();
      // [K; Q] K^T = A_hi B_hi + A_hi B_lo + A_lo B_hi (B = the K rows of A).
      const uint32_t idesc = dev::idesc_f16_f32(128, 64, 0, 0);
      const uint64_t hi = dev::sdesc_sw128(sbase, 16, 1024);
      const uint64_t lo = dev::sdesc_sw128(sbase + 4 * kTile, 16, 1024);
      const uint64_t pa[3] = {hi, hi, lo}, pb[3] = {hi, lo, hi};
#pragma unroll
      for (int t = 0; t < 3; ++t)
#pragma unroll
        for (int ks = 0; ks < kDim / 16; ++ks) {
          const uint64_t off = uint64_t(((ks >> 2) * 2 * kTile + (ks & 3) * 32) >> 4);
          dev::tc_mma_f16_ss(tmem, pa[t] + off, pb[t] + off, idesc, (t | ks) != 0);
        }
    } else {
      *fail = 1;
    }
    dev::tc_commit(dev::smem_u32(&bars[1]));  // also arrives when nothing was issued
  }
  __syncthreads();
  const bool ok = dev::mbar_wait(dev::smem_u32(&bars[1]), 0, 0x31) &&
                  !*reinterpret_cast<volatile int*>(fail);
  dev::tc_fence_after();
  if (__all_sync(0xffffffffu, ok)) {
    // Row r of the product: r < 64: k_r . k_j; r >= 64: q_(r-64) . k_j.
    const unsigned r = tid;
    uint32_t x[64];
    {
      uint32_t (&x0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&x[0]);
      uint32_t (&x1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&x[32]);
      dev::tmem_ld32(tmem + ((32u * warp) << 16), x0);
      dev::tmem_ld32(tmem + ((32u * warp) << 16) + 32, x1);
      dev::tmem_wait_ld();
    }
    if (r < kC) {
      const unsigned i = r;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float gi = gs[hh * kC + i], bi = bs[hh * kC + i];
        float* row = Ls + (hh * kC + i) * kLRow;
#pragma unroll
        for (int j = 0; j < kC; ++j)
          row[j] = j < int(i) ? bi * __expf(gi - gs[hh * kC + j]) * __uint_as_float(x[j]) : 0.0f;
      }
    } else {
      const unsigned i = r - kC;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const unsigned h = kh + kKHeads * hh;
        const float gi = gs[hh * kC + i];
        const size_t row = ((size_t(h) * a.nc + c) * kC + i) * kC;
        uint4* dst = reinterpret_cast<uint4*>(a.aqk + row);
        uint4* dstl = reinterpret_cast<uint4*>(a.aqklo + row);
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = 8 * q8 + e;
            v[e] = j <= int(i) ? __expf(gi - gs[hh * kC + j]) * __uint_as_float(x[j]) : 0.0f;
          }
          uint2 h0, l0, h1, l1;
          const float v0[4] = {v[0], v[1], v[2], v[3]}, v1[4] = {v[4], v[5], v[6], v[7]};
          split4(v0, h0, l0);
          split4(v1, h1, l1);
          dst[q8] = make_uint4(h0.x, h0.y, h1.x, h1.y);
          dstl[q8] = make_uint4(l0.x, l0.y, l1.x, l1.y);
        }
      }
    }
  }
  dev::tc_fence_before();
  __syncthreads();
  // T = (I + L)^-1 by forward substitution, thread (hh, col) solving column col of V head
  // kh + 16 hh: t_i = [i == col] - sum_{j<i} L_ij t_j. Rows go in blocks of 16: first the
  // contributions of all earlier rows to the block's 16 rows (16 independent accumulators), then
  // the block's own 16 x 16 triangle. Solved columns live in shared memory (Tc, in the [K; Q]
  // tile area, free once the MMA has completed), which keeps the code compact.
  float* Tc = reinterpret_cast<float*>(smem);  // [2][64 cols][kTRow]
  float* fac = Tc + 2 * kC * kTRow;            // [2][2][64]: beta e^g (Tw), beta (Tu) per column
  if (ok) {
    const unsigned hh = tid / kC, col = tid % kC;
    const float* L = Ls + hh * kC * kLRow;
    float* tcol = Tc + (hh * kC + col) * kTRow;
    const float bc = bs[hh * kC + col];
    fac[(hh * 2 + 0) * kC + col] = bc * __expf(gs[hh * kC + col]);
    fac[(hh * 2 + 1) * kC + col] = bc;
#pragma unroll 1
    for (int b = 0; b < kC / 16; ++b) {
      const int i0 = 16 * b;
      float acc[16];
#pragma unroll
      for (int r = 0; r < 16; ++r)
        acc[r] = i0 + r == int(col) ? 1.0f : 0.0f;
#pragma unroll 1
      for (int j = 0; j < i0; j += 4) {
        const float t0 = tcol[j], t1 = tcol[j + 1], t2 = tcol[j + 2], t3 = tcol[j + 3];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const float4 l4 = *reinterpret_cast<const float4*>(L + (i0 + r) * kLRow + j);
          acc[r] -= l4.x * t0 + l4.y * t1 + l4.z * t2 + l4.w * t3;
        }
      }
#pragma unroll
      for (int r = 1; r < 16; ++r)
#pragma unroll
        for (int q = 0; q < r; ++q)
          acc[r] -= L[(i0 + r) * kLRow + i0 + q] * acc[q];
#pragma unroll
      for (int r = 0; r < 16; ++r)
        tcol[i0 + r] = acc[r];
    }
  }
  __syncthreads();
  if (ok) {
    // Tw = T diag(beta e^g), Tu = T diag(beta) as fp16 rows: 16-byte chunk (hh, which, i, k)
    // holds columns 8k .. 8k + 7 of row i.
    for (unsigned u = tid; u < 2 * 2 * kC * 8; u += kPrepThreads) {
      const unsigned k = u % 8, i = (u / 8) % kC, which = (u / (8 * kC)) % 2, hh = u / (16 * kC);
      const float* f = fac + (hh * 2 + which) * kC + 8 * k;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        v[e] = Tc[(hh * kC + 8 * k + e) * kTRow + i] * f[e];
      const unsigned h = kh + kKHeads * hh;
      __half* dst = (which ? a.tu : a.tw) + ((size_t(h) * a.nc + c) * kC + i) * kC + 8 * k;
      *reinterpret_cast<uint4*>(dst) =
          make_uint4(h2(v[0], v[1]), h2(v[2], v[3]), h2(v[4], v[5]), h2(v[6], v[7]));
    }
  }
  if (tid == 0 && *reinterpret_cast<volatile int*>(fail))
    dev::mbar_wait(dev::smem_u32(&bars[0]), 0, 0x31);  // let the tile copies land (bounded)
  __syncthreads();
  if (warp == 0) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, 64);
  }
}

// =============================================================================== recur_kernel

struct RecurArgs {
  const float* eg;      // [32][np] e^(g_t)
  const float* egl;     // [32][np] e^(g_last - g_t)
  const float* z;       // z[t * zab_stride + h * 128 + v]
  const float* norm_w;  // [128]
  float* state;         // [32][128 k][128 v]
  float* out;           // [n][4096]
  unsigned n, np, nc, zab_stride;
  unsigned z_prefetch;  // z rows are 16-byte aligned: the producer prefetches them into L2
  float eps;
};

constexpr int kRecurThreads = 512;  // warp 0 TMA, warp 1 MMA + TMEM, 4-11 state, 12-15 output
// Stage (double-buffered, one chunk): K, Q as [64 tokens][128] fp16 in two 64-column boxes
// each, Aqk high part and remainder as [64][64] fp16. The state warps scale the K rows by
// e^(g_last - g_j) and the Q rows by e^(g_i) in place once W^T has been computed from K.
constexpr uint32_t kStK = 0, kStQ = 2 * kTile, kStAh = 4 * kTile, kStAl = 5 * kTile,
                   kStageBytes = 6 * kTile;  // 48 KB
// Inputs of W^T and U^T (single-buffered, reloaded as soon as the MMAs of a chunk consumed them):
// V high part and remainder [64][128] fp16, Tw and Tu [64][64] fp16.
constexpr uint32_t kOffP1 = 2 * kStageBytes;
constexpr uint32_t kP1Vh = 0, kP1Vl = 2 * kTile, kP1Tw = 4 * kTile, kP1Tu = 5 * kTile,
                   kP1Bytes = 6 * kTile;  // 48 KB
constexpr uint32_t kOffS16 = kOffP1 + kP1Bytes;    // S^T fp16, two 16 KB column slabs
constexpr uint32_t kOffW16 = kOffS16 + 4 * kTile;  // W^T fp16 [k][i] (MN-major B)
constexpr uint32_t kOffDh = kOffW16 + 2 * kTile;   // delta^T fp16 [v][j], high part
constexpr uint32_t kOffDl = kOffDh + 2 * kTile;    // and remainder
constexpr uint32_t kOffRed = kOffDl + 2 * kTile;   // [2][4 warps][64] fp32
constexpr uint32_t kOffBar = kOffRed + 2 * 4 * kC * 4;

struct RecurBars {
  uint64_t stage_full[2], stage_empty[2], p1in_full, p1in_empty;
  uint64_t p1_full, ut_full[2], w16_ready, kq_ready, s16_ready, s_scaled, x_full, d_ready, s_full;
  uint64_t o_full[2], o_free[2], red_ready[2], drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t kRecurSmemBytes = kOffBar + sizeof(RecurBars);
static_assert(kRecurSmemBytes <= 232448, "fits the 227 KB opt-in shared memory");

// TMEM columns (lane = row of the M = 128 tiles). O and U^T are double-buffered by chunk parity.
constexpr uint32_t kColS = 0, kColX = 128, kColO = 192, kColWt = 320, kColUt = 384;

__device__ __forceinline__ bool aborted(const RecurBars& b) {
  return *reinterpret_cast<const volatile int*>(&b.abort_flag) != 0;
}

__device__ __forceinline__ bool wait_or_abort(RecurBars& b, uint64_t& bar, uint32_t parity) {
  if (aborted(b))
    return false;
  if (!dev::mbar_wait(dev::smem_u32(&bar), parity, 0x30)) {
    b.abort_flag = 1;
    return false;
  }
  return true;
}

// Warp-collective bounded wait: every lane waits, the warp proceeds only if all succeeded.
__device__ __forceinline__ bool warp_wait(RecurBars& b, uint64_t& bar, uint32_t parity) {
  return __all_sync(0xffffffffu, wait_or_abort(b, bar, parity));
}

__device__ __forceinline__ void warp_arrive(uint64_t& bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0)
    dev::mbar_arrive(dev::smem_u32(&bar));
}

// Eight fp32 values as one 16-byte chunk of fp16.
__device__ __forceinline__ uint4 pack8(const float* v) {
  return make_uint4(h2(v[0], v[1]), h2(v[2], v[3]), h2(v[4], v[5]), h2(v[6], v[7]));
}

// Eight fp32 values as fp16 high parts and remainders (two 16-byte chunks).
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
  uint2 h0, l0, h1, l1;
  const float a[4] = {v[0], v[1], v[2], v[3]}, b[4] = {v[4], v[5], v[6], v[7]};
  split4(a, h0, l0);
  split4(b, h1, l1);
  hi = make_uint4(h0.x, h0.y, h1.x, h1.y);
  lo = make_uint4(l0.x, l0.y, l1.x, l1.y);
}

// Scales the eight fp16 values of a 16-byte chunk by f (in place).
__device__ __forceinline__ void scale8(uint4* p, float f) {
  uint4 w = *p;
  __half2* h = reinterpret_cast<__half2*>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 x = __half22float2(h[e]);
    h[e] = __floats2half2_rn(x.x * f, x.y * f);
  }
  *p = w;
}

__global__ void __launch_bounds__(kRecurThreads, 1)
    recur_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                 const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap vlmap,
                 const __grid_constant__ CUtensorMap twmap, const __grid_constant__ CUtensorMap tumap,
                 const __grid_constant__ CUtensorMap aqkmap,
                 const __grid_constant__ CUtensorMap aqklmap, RecurArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((dev::smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0)
      dev::set_status(dev::kStatusTimeout, 0x30);
    return;
  }
  RecurBars& bar = *reinterpret_cast<RecurBars*>(smem + kOffBar);
  const unsigned h = blockIdx.x, kh = h % kKHeads, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const unsigned nc = a.nc;
  const uint32_t sbase = dev::smem_u32(smem);
  const float* egh = a.eg + size_t(h) * a.np;
  const float* eglh = a.egl + size_t(h) * a.np;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(dev::smem_u32(&bar.stage_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.stage_empty[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.ut_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.o_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.o_free[s]), 4);
      dev::mbar_init(dev::smem_u32(&bar.red_ready[s]), 4);
    }
    dev::mbar_init(dev::smem_u32(&bar.p1in_full), 1);
    dev::mbar_init(dev::smem_u32(&bar.p1in_empty), 1);
    dev::mbar_init(dev::smem_u32(&bar.p1_full), 1);
    dev::mbar_init(dev::smem_u32(&bar.w16_ready), 8);
    dev::mbar_init(dev::smem_u32(&bar.kq_ready), 8);
    dev::mbar_init(dev::smem_u32(&bar.s16_ready), 8);
    dev::mbar_init(dev::smem_u32(&bar.s_scaled), 8);
    dev::mbar_init(dev::smem_u32(&bar.x_full), 1);
    dev::mbar_init(dev::smem_u32(&bar.d_ready), 8);
    dev::mbar_init(dev::smem_u32(&bar.s_full), 1);
    dev::mbar_init(dev::smem_u32(&bar.drain), 1);
    bar.abort_flag = 0;
    dev::mbar_init_fence();
  }
  if (warp == 1) {
    dev::tmem_alloc(dev::smem_u32(&bar.tmem_base), 512);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------------------ producer
    if (lane == 0) {
      dev::tma_prefetch_desc(&qmap);
      dev::tma_prefetch_desc(&kmap);
      dev::tma_prefetch_desc(&vmap);
      unsigned staged = 0, p1in = 0;  // chunks whose stage / W-U inputs have been issued
      for (unsigned c = 0; c < nc; ++c) {
        const unsigned s = c & 1;
        if (c >= 2 && !wait_or_abort(bar, bar.stage_empty[s], ((c >> 1) & 1) ^ 1))
          break;
        const uint32_t sb = sbase + s * kStageBytes, full = dev::smem_u32(&bar.stage_full[s]);
        dev::mbar_arrive_expect_tx(full, kStageBytes);
        for (int x = 0; x < 2; ++x) {
          dev::tma_load_3d(sb + kStK + x * kTile, &kmap, x * 64, kh, c * kC, full);
          dev::tma_load_3d(sb + kStQ + x * kTile, &qmap, x * 64, kh, c * kC, full);
        }
        const int row = int((h * nc + c) * kC);
        dev::tma_load_2d(sb + kStAh, &aqkmap, 0, row, full);
        dev::tma_load_2d(sb + kStAl, &aqklmap, 0, row, full);
        staged = c + 1;
        if (c >= 1 && !wait_or_abort(bar, bar.p1in_empty, (c - 1) & 1))
          break;
        const uint32_t pb = sbase + kOffP1, pfull = dev::smem_u32(&bar.p1in_full);
        dev::mbar_arrive_expect_tx(pfull, kP1Bytes);
        for (int x = 0; x < 2; ++x) {
          dev::tma_load_3d(pb + kP1Vh + x * kTile, &vmap, x * 64, h, c * kC, pfull);
          dev::tma_load_3d(pb + kP1Vl + x * kTile, &vlmap, x * 64, h, c * kC, pfull);
        }
        dev::tma_load_2d(pb + kP1Tw, &twmap, 0, row, pfull);
        dev::tma_load_2d(pb + kP1Tu, &tumap, 0, row, pfull);
        p1in = c + 1;
        if (a.z_prefetch) {  // this chunk's gate rows (512 B each) into L2 for the output warps
          for (unsigned i = 0; i < kC && c * kC + i < a.n; ++i)
            dev::prefetch_l2(a.z + size_t(c * kC + i) * a.zab_stride + h * kDim, kDim * 4);
        }
      }
      if (aborted(bar)) {  // let the copies already issued land before the CTA exits (bounded)
        for (unsigned c = staged >= 2 ? staged - 2 : 0; c < staged; ++c)
          dev::mbar_wait(dev::smem_u32(&bar.stage_full[c & 1]), (c >> 1) & 1);
        if (p1in > 0)
          dev::mbar_wait(dev::smem_u32(&bar.p1in_full), (p1in - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t id_x = dev::idesc_f16_f32(128, 64, 0, 1);   // S^T . W^T   (B MN-major)
      const uint32_t id_y = dev::idesc_f16_f32(128, 64, 0, 0);   // S^T . Qg^T
      const uint32_t id_p = dev::idesc_f16_f32(128, 64, 1, 0);   // K^T . Tw^T  (A MN-major)
      const uint32_t id_s = dev::idesc_f16_f32(128, 128, 0, 1);  // delta^T . Ks
      const uint32_t id_z = dev::idesc_f16_f32(128, 64, 0, 0);   // delta^T . Aqk^T
      auto kdesc = [](uint32_t addr) { return dev::sdesc_sw128(addr, 16, 1024); };
      auto mdesc = [](uint32_t addr) { return dev::sdesc_sw128(addr, kTile, 1024); };
      // W^T = K^T Tw^T and U^T = (V_hi + V_lo)^T Tu^T of chunk c.
      auto issue_p1 = [&](unsigned c) {
        const uint32_t sb = sbase + (c & 1) * kStageBytes, pb = sbase + kOffP1;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          dev::tc_mma_f16_ss(tmem + kColWt, mdesc(sb + kStK + kk * 2048),
                             kdesc(pb + kP1Tw + kk * 32), id_p, kk > 0);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            dev::tc_mma_f16_ss(tmem + kColUt + 64 * (c & 1),
                               mdesc(pb + (t ? kP1Vl : kP1Vh) + kk * 2048),
                               kdesc(pb + kP1Tu + kk * 32), id_p, (t | kk) != 0);
        dev::tc_commit(dev::smem_u32(&bar.p1_full));
        dev::tc_commit(dev::smem_u32(&bar.ut_full[c & 1]));
        dev::tc_commit(dev::smem_u32(&bar.p1in_empty));
      };
      bool ok = wait_or_abort(bar, bar.stage_full[0], 0) && wait_or_abort(bar, bar.p1in_full, 0);
      if (ok) {
        dev::tc_fence_after();
        issue_p1(0);
      }
      for (unsigned c = 0; ok && c < nc; ++c) {
        const unsigned b = c & 1;
        const uint32_t sb = sbase + b * kStageBytes, ocol = tmem + kColO + 64 * b;
        if (!wait_or_abort(bar, bar.s16_ready, c & 1) || !wait_or_abort(bar, bar.w16_ready, c & 1))
          break;
        dev::tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          dev::tc_mma_f16_ss(tmem + kColX,
                             kdesc(sbase + kOffS16 + (ks >> 2) * 2 * kTile + (ks & 3) * 32),
                             mdesc(sbase + kOffW16 + ks * 2048), id_x, ks > 0);
        dev::tc_commit(dev::smem_u32(&bar.x_full));
        // The scaled K / Q of this chunk (and W^T read from the unscaled K) must be in place
        // before the next chunk's W^T / U^T are issued, so that the state warps' next kq_ready
        // arrival cannot run ahead of this wait.
        if (!wait_or_abort(bar, bar.kq_ready, c & 1))
          break;
        if (c + 1 < nc) {
          if (!wait_or_abort(bar, bar.stage_full[(c + 1) & 1], ((c + 1) >> 1) & 1) ||
              !wait_or_abort(bar, bar.p1in_full, (c + 1) & 1))
            break;
          dev::tc_fence_after();
          issue_p1(c + 1);
        }
        if (c >= 2 && !wait_or_abort(bar, bar.o_free[b], ((c >> 1) & 1) ^ 1))
          break;
        dev::tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          dev::tc_mma_f16_ss(ocol, kdesc(sbase + kOffS16 + (ks >> 2) * 2 * kTile + (ks & 3) * 32),
                             kdesc(sb + kStQ + (ks >> 2) * kTile + (ks & 3) * 32), id_y, ks > 0);
        if (!wait_or_abort(bar, bar.d_ready, c & 1) || !wait_or_abort(bar, bar.s_scaled, c & 1))
          break;
        dev::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          dev::tc_mma_f16_ss(tmem + kColS, kdesc(sbase + kOffDh + kk * 32),
                             mdesc(sb + kStK + kk * 2048), id_s, 1);
        dev::tc_commit(dev::smem_u32(&bar.s_full));
        // O += D_hi A_hi + D_hi A_lo + D_lo A_hi
        const uint32_t za[3] = {kOffDh, kOffDh, kOffDl}, zb[3] = {kStAh, kStAl, kStAh};
#pragma unroll
        for (int t = 0; t < 3; ++t)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            dev::tc_mma_f16_ss(ocol, kdesc(sbase + za[t] + kk * 32), kdesc(sb + zb[t] + kk * 32),
                               id_z, 1);
        dev::tc_commit(dev::smem_u32(&bar.o_full[b]));
        dev::tc_commit(dev::smem_u32(&bar.stage_empty[b]));
      }
      dev::tc_commit(dev::smem_u32(&bar.drain));
      dev::mbar_wait(dev::smem_u32(&bar.drain), 0);
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------- state warps: S^T copies, delta^T, W^T to fp16, K / Q scaling
    // Warp (4 + q + 4 hc): TMEM lanes [32 q, 32 q + 32) (rows v of S^T, X, U; rows k of W^T);
    // S^T columns (k) [64 hc, +64), X / U / W^T columns [32 hc, +32).
    const unsigned q = warp & 3, hc = (warp - 4) >> 2, v = 32 * q + lane;
    const unsigned st = threadIdx.x - 128;  // 0..255
    const uint32_t trow = tmem + ((32u * q) << 16);
    uint8_t* s16 = smem + kOffS16 + hc * 2 * kTile + v * 128;
    uint8_t* dh16 = smem + kOffDh + v * 128;
    uint8_t* dl16 = smem + kOffDl + v * 128;
    uint8_t* w16 = smem + kOffW16 + v * 128;  // row k = v of W^T
    const float* S = a.state + size_t(h) * kDim * kDim;
    // EW(c): W^T of chunk c (TMEM, fp32) -> fp16 rows [k][i] of W16, the MN-major B operand of
    // X(c); then, W^T having consumed the unscaled K, the K rows of the stage are scaled by
    // e^(g_last - g_j) (the state update's decay) and the Q rows by e^(g_i) (the output's).
    // W16 is free: X(c - 1) has completed (E1(c - 1) waited for it).
    auto ew = [&](unsigned c) -> bool {
      const unsigned r0 = st / 8, r1 = r0 + 32;  // the two tile rows this thread rescales
      const float fk0 = eglh[c * kC + r0], fk1 = eglh[c * kC + r1];
      const float fq0 = egh[c * kC + r0], fq1 = egh[c * kC + r1];
      if (!warp_wait(bar, bar.p1_full, c & 1) ||
          !warp_wait(bar, bar.stage_full[c & 1], (c >> 1) & 1))
        return false;
      dev::tc_fence_after();
      uint32_t x[32];
      dev::tmem_ld32(trow + kColWt + 32 * hc, x);
      dev::tmem_wait_ld();
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          f[e] = __uint_as_float(x[8 * cc + e]);
        *reinterpret_cast<uint4*>(w16 + (((4 * hc + cc) ^ (v & 7)) << 4)) = pack8(f);
      }
      dev::fence_proxy_async_smem();
      dev::tc_fence_before();
      warp_arrive(bar.w16_ready);
      // 16-byte chunk u = st + 256 m of a [64 rows][128 B] x 2 box tile lies in row (u % 512) / 8.
      uint4* kt = reinterpret_cast<uint4*>(smem + (c & 1) * kStageBytes + kStK);
      uint4* qt = reinterpret_cast<uint4*>(smem + (c & 1) * kStageBytes + kStQ);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        scale8(kt + st + 256 * m, (m & 1) ? fk1 : fk0);
        scale8(qt + st + 256 * m, (m & 1) ? fq1 : fq0);
      }
      dev::fence_proxy_async_smem();
      warp_arrive(bar.kq_ready);
      return true;
    };
    bool ok = ew(0);
    for (unsigned c = 0; ok && c < nc; ++c) {
      const float el = egh[c * kC + kC - 1];  // e^(g_last)
      // E0: fp16 copy of S^T for X / Y, then S^T *= e^(g_last) in TMEM for the update MMA.
      if (c > 0 && !warp_wait(bar, bar.s_full, (c - 1) & 1)) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const uint32_t col = kColS + 64 * hc + 32 * half;
        uint32_t x[32];
        if (c == 0) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            x[e] = __float_as_uint(S[size_t(64 * hc + 32 * half + e) * kDim + v]);
        } else {
          dev::tmem_ld32(trow + col, x);
          dev::tmem_wait_ld();
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            f[e] = __uint_as_float(x[8 * cc + e]);
          *reinterpret_cast<uint4*>(s16 + (((4 * half + cc) ^ (v & 7)) << 4)) = pack8(f);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e)
          x[e] = __float_as_uint(__uint_as_float(x[e]) * el);
        dev::tmem_st32(trow + col, x);
      }
      dev::fence_proxy_async_smem();
      warp_arrive(bar.s16_ready);
      dev::tmem_wait_st();
      dev::tc_fence_before();
      warp_arrive(bar.s_scaled);

      // E1: delta^T = U^T - X^T as fp16 high part and remainder.
      if (!warp_wait(bar, bar.x_full, c & 1) ||
          !warp_wait(bar, bar.ut_full[c & 1], (c >> 1) & 1)) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
      uint32_t xx[32], uu[32];
      dev::tmem_ld32(trow + kColX + 32 * hc, xx);
      dev::tmem_ld32(trow + kColUt + 64 * (c & 1) + 32 * hc, uu);
      dev::tmem_wait_ld();
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float d[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          d[e] = __uint_as_float(uu[8 * cc + e]) - __uint_as_float(xx[8 * cc + e]);
        uint4 hi, lo;
        split8(d, hi, lo);
        const unsigned chunk = ((4 * hc + cc) ^ (v & 7)) << 4;
        *reinterpret_cast<uint4*>(dh16 + chunk) = hi;
        *reinterpret_cast<uint4*>(dl16 + chunk) = lo;
      }
      dev::fence_proxy_async_smem();
      dev::tc_fence_before();
      warp_arrive(bar.d_ready);
      if (c + 1 < nc && !ew(c + 1)) {
        ok = false;
        break;
      }
    }
    // Final state back to [k][v] (coalesced over v).
    if (ok && warp_wait(bar, bar.s_full, (nc - 1) & 1)) {
      dev::tc_fence_after();
      float* So = a.state + size_t(h) * kDim * kDim;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t x[32];
        dev::tmem_ld32(trow + kColS + 64 * hc + 32 * half, x);
        dev::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          So[size_t(64 * hc + 32 * half + e) * kDim + v] = __uint_as_float(x[e]);
      }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------ output warps: RMS norm, gate, store
    // Thread = value column v of the head. O^T[v][i] of chunk c is read from TMEM twice: once for
    // the sums of squares (reduced over v), then eight tokens at a time for the outputs. The 64
    // gate inputs of the chunk are loaded before O is waited for, and the per-token arithmetic
    // is branch-free (one warp-uniform bound check per group of eight), so the dependent
    // latencies of the eight tokens overlap.
    const unsigned q = warp & 3, v = 32 * q + lane;
    const uint32_t trow = tmem + ((32u * q) << 16);
    float* red = reinterpret_cast<float*>(smem + kOffRed);
    const float nw = a.norm_w[v];
    const float* zh = a.z + h * kDim + v;
    float* oh = a.out + h * kDim + v;
    constexpr int kG = 8;
    for (unsigned c = 0; c < nc; ++c) {
      const unsigned b = c & 1, t0 = c * kC;
      const uint32_t ocol = trow + kColO + 64 * b;
      const unsigned last = a.n - 1 - t0;  // tokens past the end read token n - 1's gate (unused)
      float zr[kC];
#pragma unroll
      for (int i = 0; i < kC; ++i)
        zr[i] = zh[size_t(t0 + min(unsigned(i), last)) * a.zab_stride];
      if (!warp_wait(bar, bar.o_full[b], (c >> 1) & 1))
        break;
      dev::tc_fence_after();
      float* rb = red + b * 4 * kC;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t x[32];
        dev::tmem_ld32(ocol + 32 * half, x);
        dev::tmem_wait_ld();
        float s2[32];
#pragma unroll
        for (int e = 0; e < 32; ++e)
          s2[e] = __uint_as_float(x[e]) * __uint_as_float(x[e]);
        // Reduce-scatter over the warp: lane l ends with token 32 half + l.
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
          const bool upper = (lane & off) != 0;
#pragma unroll
          for (int k = 0; k < off; ++k) {
            const float send = upper ? s2[k] : s2[k + off];
            const float keep = upper ? s2[k + off] : s2[k];
            s2[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
          }
        }
        rb[q * kC + 32 * half + lane] = s2[0];
      }
      // Exchange through an mbarrier (bounded wait), so a warp that gave up cannot strand the
      // others. Buffer b is rewritten only after every warp has passed the next chunk's wait,
      // i.e. has finished reading it.
      warp_arrive(bar.red_ready[b]);
      if (!warp_wait(bar, bar.red_ready[b], (c >> 1) & 1))
        break;
      // 1 / rms of tokens lane and 32 + lane, shared across the warp by shuffles below.
      const float r_lo = rsqrtf((rb[lane] + rb[kC + lane] + rb[2 * kC + lane] + rb[3 * kC + lane]) *
                                    (1.0f / kDim) + a.eps);
      const float r_hi = rsqrtf((rb[32 + lane] + rb[kC + 32 + lane] + rb[2 * kC + 32 + lane] +
                                 rb[3 * kC + 32 + lane]) * (1.0f / kDim) + a.eps);
#pragma unroll
      for (int g = 0; g < kC / kG; ++g) {
        uint32_t x[kG];
        dev::tmem_ld8(ocol + kG * g, x);
        dev::tmem_wait_ld();
        float y[kG];
#pragma unroll
        for (int e = 0; e < kG; ++e) {
          const int i = kG * g + e;
          const float r = __shfl_sync(0xffffffffu, i < 32 ? r_lo : r_hi, i & 31);
          y[e] = __uint_as_float(x[e]) * r * nw * silu_fast(zr[i]);
        }
        float* dst = oh + size_t(t0 + kG * g) * kVHeads * kDim;
        if (t0 + kG * g + kG <= a.n) {
#pragma unroll
          for (int e = 0; e < kG; ++e)
            dst[size_t(e) * kVHeads * kDim] = y[e];
        } else {
#pragma unroll
          for (int e = 0; e < kG; ++e)
            if (t0 + kG * g + e < a.n)
              dst[size_t(e) * kVHeads * kDim] = y[e];
        }
      }
      dev::tc_fence_before();
      warp_arrive(bar.o_free[b]);
    }
  }

  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, 512);
  }
}

}  // namespace miso::fast::dnchunk
