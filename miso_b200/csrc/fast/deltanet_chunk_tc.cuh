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
//                   high parts and fp16 remainders, and the final conv history.
//   prepare_kernel  one block per (chunk, K head), both V heads of the K head: everything of the
//                   chunk that does not depend on the state. [K; Q] K^T as one tcgen05 MMA
//                   (M=128, N=64, K=128) over hi / lo operands, L and Aqk from it, T = (I + L)^-1
//                   by blocked forward substitution, then W = [Tw_0; Tw_1] K for both V heads as
//                   one M=128 MMA; writes W, Ks = K rows * e^(g_last - g), Qg = Q rows * e^g,
//                   Tu = T diag(beta), Aqk (hi + lo) as fp16 tiles and e^g.
//   recur_kernel    one block per V head (640 threads), the 128 x 128 state transposed (S^T:
//                   lane = v, column = k) as an fp32 TMEM accumulator; per chunk, tcgen05 MMA
//                   groups with M = 128 whose A operands (S^T, delta^T as fp16) live in TMEM:
//                     [X^T | O^T] = S^T [W; Qg]^T                  (one N = 128 product)
//                     U^T = (V_hi + V_lo)^T Tu^T                   (one chunk ahead)
//                     S^T += delta^T Ks,  O^T += delta^T Aqk^T     (delta, Aqk as hi + lo)
//                   and the CUDA-core epilogues delta^T = U^T - X^T and the gated RMS norm of O.
//
// Precision: every MMA accumulates in fp32 and the state stays fp32 in TMEM. The products whose
// rounding reaches the outputs through cancelling sums (q . k, Aqk delta, U) use two-term fp16
// operands (hi + lo), the others plain fp16 (W, Ks, Qg and the S^T copy are rounded once from
// fp32); outputs stay within ~1e-4 relative (~6e-3 absolute at 8192 tokens) of an fp64
// recurrence.
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
  unsigned t_begin;  // first token of this launch (a multiple of 16; the grid covers the rest)
};

constexpr int kConvThreads = 256;
constexpr int kConvTokens = 16;  // tokens per block: the block's conv weights are read once

// Block (m, y): channels [1024 m, 1024 m + 1024) of tokens [16 y, 16 y + 16). Thread t owns the
// four channels 1024 m + 4 t .. + 3, so a warp covers one whole 128-channel head (m = 0, 1: q
// heads; 2, 3: k heads; 4..7: v heads) and the q / k L2 norms are warp reductions. The 4-tap
// window slides along the block's tokens in registers.
__global__ void __launch_bounds__(kConvThreads) conv_kernel(ConvArgs a) {
  const unsigned m = blockIdx.x, t0 = a.t_begin + blockIdx.y * kConvTokens, tid = threadIdx.x,
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
  __half* w;          // [32][nc][64][128] W = T diag(beta e^g) K
  __half* ks;         // [32][nc][64][128] K rows * e^(g_last - g_j)
  __half* qg;         // [32][nc][64][128] Q rows * e^(g_i)
  __half* tu;         // [32][nc][64][64] T diag(beta)
  __half* aqk;        // [32][nc][64][64] Aqk as fp16 high part ...
  __half* aqklo;      // ... and fp16 remainder
  unsigned n, np, nc;
  unsigned c_begin;  // first chunk of this launch (block x = chunk - c_begin)
};

constexpr int kPrepThreads = 128;
constexpr int kLRow = 68;  // fp32 row stride of L (16-byte aligned rows)
// [K; Q] as fp16 high parts (32 KB) then remainders (32 KB): 64-dim slab s of part p at
// 32 KB p + 16 KB s, K rows first, Q rows 8 KB later (M = 128 rows).
constexpr uint32_t kPrepOffL = 8 * kTile;
constexpr uint32_t kPrepOffG = kPrepOffL + 2 * kC * kLRow * 4;  // g, beta, fac, e^g, e^(gl-g)
constexpr uint32_t kPrepOffBar = kPrepOffG + 12 * kC * 4;
constexpr size_t kPrepSmemBytes = kPrepOffBar + 64;
// Solved T (fp32 [2 heads][64 rows i][64 columns j]) reuses the remainder half of the tile area,
// and [Tw_0; Tw_1] (fp16 [128 rows][64], 128-byte swizzled, the A operand of W) the L area.
static_assert(2 * kC * kC * 4 <= 4 * kTile, "T fits in the remainder tiles");
static_assert(2 * kTile <= 2 * kC * kLRow * 4, "[Tw_0; Tw_1] fits in the L area");

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
  const unsigned c = a.c_begin + blockIdx.x, kh = blockIdx.y, tid = threadIdx.x, warp = tid / 32,
                 lane = tid % 32;
  const uint32_t sbase = dev::smem_u32(smem);
  float* Ls = reinterpret_cast<float*>(smem + kPrepOffL);  // [2][64][kLRow]
  float* gs = reinterpret_cast<float*>(smem + kPrepOffG);  // [2][64]
  float* bs = gs + 2 * kC;                                 // [2][64] beta
  float* fac = bs + 2 * kC;                                // [2][2][64] beta e^g, beta
  float* egs = fac + 4 * kC;                               // [2][64] e^g
  float* egls = egs + 2 * kC;                              // [2][64] e^(g_last - g)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPrepOffBar);  // load, KK^T, W
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  int* fail = reinterpret_cast<int*>(bars + 4);

  if (tid == 0) {
    for (int i = 0; i < 3; ++i)
      dev::mbar_init(dev::smem_u32(&bars[i]), 1);
    *fail = 0;
    dev::mbar_init_fence();
  }
  if (warp == 0) {
    dev::tmem_alloc(dev::smem_u32(tmem_slot), 128);
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
    const unsigned i0 = warp * kC + 2 * lane;
    gs[i0] = g0;
    gs[i0 + 1] = g1;
    bs[i0] = t0 < a.n ? a.beta[size_t(h) * a.np + t0] : 0.0f;
    bs[i0 + 1] = t0 + 1 < a.n ? a.beta[size_t(h) * a.np + t0 + 1] : 0.0f;
    const float e0 = __expf(g0), e1 = __expf(g1);
    egs[i0] = e0;
    egs[i0 + 1] = e1;
    egls[i0] = __expf(glast - g0);
    egls[i0 + 1] = __expf(glast - g1);
    *reinterpret_cast<float2*>(a.eg + size_t(h) * a.np + t0) = make_float2(e0, e1);
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
  // the block's own 16 x 16 triangle. T is kept as [hh][i][col] (a lane's column is its bank) in
  // the remainder tiles, free once the MMA has completed; the K and Q high parts stay in place.
  float* Tc = reinterpret_cast<float*>(smem + 4 * kTile);  // [2][64 rows][64 cols]
  if (ok) {
    const unsigned hh = tid / kC, col = tid % kC;
    const float* L = Ls + hh * kC * kLRow;
    float* tcol = Tc + hh * kC * kC + col;  // row i at tcol[i * kC]
    const float bc = bs[hh * kC + col];
    fac[(hh * 2 + 0) * kC + col] = bc * egs[hh * kC + col];
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
        const float t0 = tcol[j * kC], t1 = tcol[(j + 1) * kC], t2 = tcol[(j + 2) * kC],
                    t3 = tcol[(j + 3) * kC];
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
        tcol[(i0 + r) * kC] = acc[r];
    }
  }
  __syncthreads();
  uint8_t* twt = smem + kPrepOffL;  // [Tw_0; Tw_1]: [128 rows (hh, i)][64 j] fp16, swizzled
  if (ok) {
    // Tw = T diag(beta e^g) into the swizzled A tile of W, Tu = T diag(beta) to global; 16-byte
    // chunk u: row (hh, i) = u / 8, columns 8 (u % 8) .. + 7.
#pragma unroll 2
    for (unsigned u = tid; u < 2 * kC * 8; u += kPrepThreads) {
      const unsigned cc = u % 8, r = u / 8, hh = r / kC, i = r % kC;
      const float* t = Tc + r * kC + 8 * cc;
      const float4 ta = *reinterpret_cast<const float4*>(t);
      const float4 tb = *reinterpret_cast<const float4*>(t + 4);
      const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
      const float* fw = fac + (hh * 2 + 0) * kC + 8 * cc;
      const float* fu = fac + (hh * 2 + 1) * kC + 8 * cc;
      uint32_t w4[4], u4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        w4[e] = h2(tv[2 * e] * fw[2 * e], tv[2 * e + 1] * fw[2 * e + 1]);
        u4[e] = h2(tv[2 * e] * fu[2 * e], tv[2 * e + 1] * fu[2 * e + 1]);
      }
      *reinterpret_cast<uint4*>(twt + dev::swz128(r, cc)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      const unsigned h = kh + kKHeads * hh;
      *reinterpret_cast<uint4*>(a.tu + ((size_t(h) * a.nc + c) * kC + i) * kC + 8 * cc) =
          make_uint4(u4[0], u4[1], u4[2], u4[3]);
    }
    dev::fence_proxy_async_smem();
  }
  __syncthreads();
  if (tid == 0 && ok) {
    // W = [Tw_0; Tw_1] K for both V heads in one M = 128 product: A = the Tw tile (K-major,
    // K = j), B = the K rows (MN-major, N = 128 dims in two 64-dim slabs 16 KB apart).
    dev::tc_fence_after();
    const uint32_t idesc = dev::idesc_f16_f32(128, 128, 0, 1);
    const uint32_t ta = dev::smem_u32(twt);
#pragma unroll
    for (int kk = 0; kk < kC / 16; ++kk)
      dev::tc_mma_f16_ss(tmem, dev::sdesc_sw128(ta + kk * 32, 16, 1024),
                         dev::sdesc_sw128(sbase + kk * 2048, 2 * kTile, 1024), idesc, kk > 0);
    dev::tc_commit(dev::smem_u32(&bars[2]));
  }
  if (ok) {
    // Meanwhile: Ks = K rows * e^(g_last - g_j) and Qg = Q rows * e^(g_i) of both V heads, from
    // the (unscaled) high parts. Unit u: tensor u / 1024 (K, Q), row (u / 16) % 64, 8-dim chunk
    // u % 16 (slab chunk / 8, swizzled chunk chunk % 8).
#pragma unroll 2
    for (unsigned u = tid; u < 2 * kC * 16; u += kPrepThreads) {
      const unsigned ch = u % 16, row = (u / 16) % kC, isq = u / (16 * kC);
      const uint8_t* src = smem + (ch / 8) * 2 * kTile + isq * kTile + dev::swz128(row, ch % 8);
      const uint4 raw = *reinterpret_cast<const uint4*>(src);
      const __half2* hv = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float f = (isq ? egs : egls)[hh * kC + row];
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 xv = __half22float2(hv[e]);
          o[e] = h2(xv.x * f, xv.y * f);
        }
        const unsigned h = kh + kKHeads * hh;
        __half* dst = (isq ? a.qg : a.ks) + ((size_t(h) * a.nc + c) * kC + row) * kDim + 8 * ch;
        *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  // W rows to global: thread r = (hh, i) holds row i of W_hh (TMEM lane r, 128 columns).
  if (__all_sync(0xffffffffu, ok && dev::mbar_wait(dev::smem_u32(&bars[2]), 0, 0x31))) {
    dev::tc_fence_after();
    const unsigned hh = tid / kC, i = tid % kC, h = kh + kKHeads * hh;
    uint4* dst = reinterpret_cast<uint4*>(a.w + ((size_t(h) * a.nc + c) * kC + i) * kDim);
#pragma unroll 1
    for (int part = 0; part < 4; ++part) {
      uint32_t x[32];
      dev::tmem_ld32(tmem + ((32u * warp) << 16) + 32 * part, x);
      dev::tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 4; ++q)
        dst[4 * part + q] = make_uint4(
            h2(__uint_as_float(x[8 * q]), __uint_as_float(x[8 * q + 1])),
            h2(__uint_as_float(x[8 * q + 2]), __uint_as_float(x[8 * q + 3])),
            h2(__uint_as_float(x[8 * q + 4]), __uint_as_float(x[8 * q + 5])),
            h2(__uint_as_float(x[8 * q + 6]), __uint_as_float(x[8 * q + 7])));
    }
  }
  if (tid == 0 && *reinterpret_cast<volatile int*>(fail))
    dev::mbar_wait(dev::smem_u32(&bars[0]), 0, 0x31);  // let the tile copies land (bounded)
  dev::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, 128);
  }
}

// =============================================================================== recur_kernel

struct RecurArgs {
  const float* eg;      // [32][np] e^(g_t)
  const float* z;       // z[t * zab_stride + h * 128 + v]
  const float* norm_w;  // [128]
  float* state;         // [32][128 k][128 v]
  float* out;           // [n][4096]
  unsigned n, np, nc, zab_stride;
  unsigned c_begin, c_end;  // chunks of this launch: the state is read at c_begin, written after
  float eps;
};

constexpr int kRecurThreads = 640;  // warp 0 TMA, warp 1 MMA + TMEM, 4-11 state, 12-19 output
// Stage (double-buffered, one chunk), 128-byte swizzled fp16 tiles:
//   B of the X / Y product: two 64-dim slabs of [128 rows][64], rows [W; Qg];
//   Ks [64 j][128] as two [64][64] boxes; Aqk high part and remainder [64 i][64 j].
constexpr uint32_t kStB = 0, kStKs = 4 * kTile, kStAh = 6 * kTile, kStAl = 7 * kTile,
                   kStageBytes = 8 * kTile;  // 64 KB
// U inputs (double-buffered): V high part and remainder [64 j][128] (two boxes each), Tu [64][64].
constexpr uint32_t kOffP1 = 2 * kStageBytes;
constexpr uint32_t kP1Vh = 0, kP1Vl = 2 * kTile, kP1Tu = 4 * kTile, kP1Bytes = 5 * kTile;  // 40 KB
constexpr uint32_t kOffRed = kOffP1 + 2 * kP1Bytes;  // [2][4 warps][64] fp32
constexpr uint32_t kOffBar = kOffRed + 2 * 4 * kC * 4;

struct RecurBars {
  uint64_t stage_full[2], stage_empty[2], p1in_full[2], p1in_empty[2];
  uint64_t ut_full[2], s16_ready, s_scaled, x_full, d_ready, s_full;
  uint64_t o_full, o_free, red_ready[2], drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t kRecurSmemBytes = kOffBar + sizeof(RecurBars);
static_assert(kRecurSmemBytes <= 232448, "fits the 227 KB opt-in shared memory");

// TMEM columns (lane = row v of the M = 128 tiles): the fp32 state S^T, its fp16 copy (A operand
// of X / Y, 2 values per column), [X^T | O^T] (one N = 128 accumulator), delta^T high part and
// remainder (A operands of the S and O updates), U^T of even and odd chunks.
constexpr uint32_t kColS = 0, kColS16 = 128, kColX = 192, kColO = 256, kColDh = 320,
                   kColDl = 352, kColUt = 384;

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

// Single-thread bounded wait that polls the barrier (mbarrier.test_wait) instead of suspending in
// try_wait: the MMA issuer resumes as soon as the phase completes, not when the suspended wait is
// next rescheduled.
__device__ __forceinline__ bool poll_or_abort(RecurBars& b, uint64_t& bar, uint32_t parity) {
  const uint32_t a = dev::smem_u32(&bar);
  if (dev::mbar_test_wait(a, parity))
    return true;
  const long long t0 = clock64();
  for (unsigned i = 1;; ++i) {
    if (dev::mbar_test_wait(a, parity))
      return true;
    if ((i & 63u) == 0) {
      if (aborted(b))
        return false;
      if (clock64() - t0 > dev::kWaitLimitCycles) {
        dev::set_status(dev::kStatusTimeout, 0x30);
        b.abort_flag = 1;
        return false;
      }
    }
  }
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

// Two fp32 values as fp16 high parts (one packed pair) and remainders (another pair).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 hv = __floats2half2_rn(x0, x1);
  const float2 f = __half22float2(hv);
  hi = *reinterpret_cast<const uint32_t*>(&hv);
  lo = h2(x0 - f.x, x1 - f.y);
}

__global__ void __launch_bounds__(kRecurThreads, 1)
    recur_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap qgmap,
                 const __grid_constant__ CUtensorMap ksmap, const __grid_constant__ CUtensorMap vmap,
                 const __grid_constant__ CUtensorMap vlmap, const __grid_constant__ CUtensorMap tumap,
                 const __grid_constant__ CUtensorMap aqkmap,
                 const __grid_constant__ CUtensorMap aqklmap, RecurArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((dev::smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0)
      dev::set_status(dev::kStatusTimeout, 0x30);
    return;
  }
  RecurBars& bar = *reinterpret_cast<RecurBars*>(smem + kOffBar);
  const unsigned h = blockIdx.x, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // Chunk c of this launch (local index, for buffer parities) is chunk c0 + c of the sequence.
  const unsigned nc = a.nc, c0 = a.c_begin, ncl = a.c_end - a.c_begin;
  const uint32_t sbase = dev::smem_u32(smem);
  const float* egh = a.eg + size_t(h) * a.np;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(dev::smem_u32(&bar.stage_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.stage_empty[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.p1in_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.p1in_empty[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.ut_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.red_ready[s]), 8);
    }
    dev::mbar_init(dev::smem_u32(&bar.o_full), 1);
    dev::mbar_init(dev::smem_u32(&bar.o_free), 8);
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
      dev::tma_prefetch_desc(&wmap);
      dev::tma_prefetch_desc(&qgmap);
      dev::tma_prefetch_desc(&vmap);
      unsigned staged = 0, p1in = 0;  // chunks whose stage / U inputs have been issued
      for (unsigned c = 0; c < ncl; ++c) {
        const unsigned s = c & 1, cg = c0 + c;
        const int row = int((h * nc + cg) * kC);
        if (c >= 2 && !wait_or_abort(bar, bar.p1in_empty[s], ((c >> 1) & 1) ^ 1))
          break;
        const uint32_t pb = sbase + kOffP1 + s * kP1Bytes, pfull = dev::smem_u32(&bar.p1in_full[s]);
        dev::mbar_arrive_expect_tx(pfull, kP1Bytes);
        for (int x = 0; x < 2; ++x) {
          dev::tma_load_3d(pb + kP1Vh + x * kTile, &vmap, x * 64, h, cg * kC, pfull);
          dev::tma_load_3d(pb + kP1Vl + x * kTile, &vlmap, x * 64, h, cg * kC, pfull);
        }
        dev::tma_load_2d(pb + kP1Tu, &tumap, 0, row, pfull);
        p1in = c + 1;
        if (c >= 2 && !wait_or_abort(bar, bar.stage_empty[s], ((c >> 1) & 1) ^ 1))
          break;
        const uint32_t sb = sbase + s * kStageBytes, full = dev::smem_u32(&bar.stage_full[s]);
        dev::mbar_arrive_expect_tx(full, kStageBytes);
        for (int x = 0; x < 2; ++x) {
          dev::tma_load_2d(sb + kStB + x * 2 * kTile, &wmap, x * 64, row, full);
          dev::tma_load_2d(sb + kStB + x * 2 * kTile + kTile, &qgmap, x * 64, row, full);
          dev::tma_load_2d(sb + kStKs + x * kTile, &ksmap, x * 64, row, full);
        }
        dev::tma_load_2d(sb + kStAh, &aqkmap, 0, row, full);
        dev::tma_load_2d(sb + kStAl, &aqklmap, 0, row, full);
        staged = c + 1;
      }
      if (aborted(bar)) {  // let the copies already issued land before the CTA exits (bounded)
        for (unsigned c = staged >= 2 ? staged - 2 : 0; c < staged; ++c)
          dev::mbar_wait(dev::smem_u32(&bar.stage_full[c & 1]), (c >> 1) & 1);
        for (unsigned c = p1in >= 2 ? p1in - 2 : 0; c < p1in; ++c)
          dev::mbar_wait(dev::smem_u32(&bar.p1in_full[c & 1]), (c >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------ MMA issue
    // Per chunk c, in issue order (the tensor pipe runs them in order):
    //   XY(c)    [X^T | O^T] = S16 [W; Qg]^T (N = 128)   after E0(c) wrote S16, O^T(c-1) was read
    //   U(c+1)   U^T = (V_hi + V_lo)^T Tu^T             (double-buffered; runs during E1(c))
    //   C2(c)    S^T += Dh Ks                          after E1(c): delta written, S scaled
    //   Z(c)     O^T += Dh Ah + Dh Al + Dl Ah          (runs during E0(c+1))
    // so the tensor pipe works on U while the state warps form delta, and on Z while they copy
    // the next state, and the chain E0 -> XY -> E1 -> C2 -> E0 never queues behind them.
    if (lane == 0) {
      const uint32_t id_xy = dev::idesc_f16_f32(128, 128, 0, 0);  // A (TMEM) . B K-major
      const uint32_t id_s = dev::idesc_f16_f32(128, 128, 0, 1);   // A (TMEM) . Ks MN-major
      const uint32_t id_z = dev::idesc_f16_f32(128, 64, 0, 0);    // A (TMEM) . Aqk K-major
      const uint32_t id_u = dev::idesc_f16_f32(128, 64, 1, 0);    // V^T MN-major . Tu K-major
      auto kdesc = [](uint32_t addr) { return dev::sdesc_sw128(addr, 16, 1024); };
      auto mdesc = [](uint32_t addr) { return dev::sdesc_sw128(addr, kTile, 1024); };
      auto issue_u = [&](unsigned c) {
        const uint32_t pb = sbase + kOffP1 + (c & 1) * kP1Bytes;
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            dev::tc_mma_f16_ss(tmem + kColUt + 64 * (c & 1),
                               mdesc(pb + (t ? kP1Vl : kP1Vh) + kk * 2048),
                               kdesc(pb + kP1Tu + kk * 32), id_u, (t | kk) != 0);
        dev::tc_commit(dev::smem_u32(&bar.ut_full[c & 1]));
        dev::tc_commit(dev::smem_u32(&bar.p1in_empty[c & 1]));
      };
      bool ok = poll_or_abort(bar, bar.p1in_full[0], 0);
      if (ok) {
        dev::tc_fence_after();
        issue_u(0);
      }
      for (unsigned c = 0; ok && c < ncl; ++c) {
        const unsigned b = c & 1;
        const uint32_t sb = sbase + b * kStageBytes;
        if (!poll_or_abort(bar, bar.stage_full[b], (c >> 1) & 1) ||
            !poll_or_abort(bar, bar.s16_ready, c & 1) ||
            (c >= 1 && !poll_or_abort(bar, bar.o_free, (c - 1) & 1)))
          break;
        dev::tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          dev::tc_mma_f16_ts(tmem + kColX, tmem + kColS16 + 8 * ks,
                             kdesc(sb + kStB + (ks >> 2) * 2 * kTile + (ks & 3) * 32), id_xy,
                             ks > 0);
        dev::tc_commit(dev::smem_u32(&bar.x_full));
        if (c + 1 < ncl) {
          if (!poll_or_abort(bar, bar.p1in_full[(c + 1) & 1], ((c + 1) >> 1) & 1))
            break;
          dev::tc_fence_after();
          issue_u(c + 1);
        }
        if (!poll_or_abort(bar, bar.d_ready, c & 1) || !poll_or_abort(bar, bar.s_scaled, c & 1))
          break;
        dev::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          dev::tc_mma_f16_ts(tmem + kColS, tmem + kColDh + 8 * kk, mdesc(sb + kStKs + kk * 2048),
                             id_s, 1);
        dev::tc_commit(dev::smem_u32(&bar.s_full));
        // O += D_hi A_hi + D_hi A_lo + D_lo A_hi
        const uint32_t za[3] = {kColDh, kColDh, kColDl}, zb[3] = {kStAh, kStAl, kStAh};
#pragma unroll
        for (int t = 0; t < 3; ++t)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            dev::tc_mma_f16_ts(tmem + kColO, tmem + za[t] + 8 * kk, kdesc(sb + zb[t] + kk * 32),
                               id_z, 1);
        dev::tc_commit(dev::smem_u32(&bar.o_full));
        dev::tc_commit(dev::smem_u32(&bar.stage_empty[b]));
      }
      dev::tc_commit(dev::smem_u32(&bar.drain));
      dev::mbar_wait(dev::smem_u32(&bar.drain), 0);
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------ state warps: S16, S decay, delta
    // Warp (4 + q + 4 hc): TMEM lanes [32 q, 32 q + 32) (rows v), S^T columns (k) [64 hc, +64),
    // X^T / U^T columns (i) [32 hc, +32).
    const unsigned q = warp & 3, hc = (warp - 4) >> 2, v = 32 * q + lane;
    const uint32_t trow = tmem + ((32u * q) << 16);
    const float* S = a.state + size_t(h) * kDim * kDim;
    bool ok = true;
    for (unsigned c = 0; ok && c < ncl; ++c) {
      const float el = egh[(c0 + c) * kC + kC - 1];  // e^(g_last)
      // E0: fp16 copy of S^T (the A operand of XY), then S^T *= e^(g_last) for the update.
      if (c > 0 && !warp_wait(bar, bar.s_full, (c - 1) & 1)) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
      uint32_t x[64];
      uint32_t (&x0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&x[0]);
      uint32_t (&x1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&x[32]);
      if (c == 0) {
#pragma unroll
        for (int e = 0; e < 64; ++e)
          x[e] = __float_as_uint(S[size_t(64 * hc + e) * kDim + v]);
      } else {
        dev::tmem_ld32(trow + kColS + 64 * hc, x0);
        dev::tmem_ld32(trow + kColS + 64 * hc + 32, x1);
        dev::tmem_wait_ld();
      }
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        uint32_t p16[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          p16[e] = h2(__uint_as_float(x[32 * part + 2 * e]),
                      __uint_as_float(x[32 * part + 2 * e + 1]));
        dev::tmem_st16(trow + kColS16 + 32 * hc + 16 * part, p16);
      }
      dev::tmem_wait_st();
      dev::tc_fence_before();
      warp_arrive(bar.s16_ready);
#pragma unroll
      for (int e = 0; e < 64; ++e)
        x[e] = __float_as_uint(__uint_as_float(x[e]) * el);
      dev::tmem_st32(trow + kColS + 64 * hc, x0);
      dev::tmem_st32(trow + kColS + 64 * hc + 32, x1);
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
      for (int part = 0; part < 2; ++part) {
        uint32_t dh[8], dl[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int i = 16 * part + 2 * e;
          split2(__uint_as_float(uu[i]) - __uint_as_float(xx[i]),
                 __uint_as_float(uu[i + 1]) - __uint_as_float(xx[i + 1]), dh[e], dl[e]);
        }
        dev::tmem_st8(trow + kColDh + 16 * hc + 8 * part, dh);
        dev::tmem_st8(trow + kColDl + 16 * hc + 8 * part, dl);
      }
      dev::tmem_wait_st();
      dev::tc_fence_before();
      warp_arrive(bar.d_ready);
    }
    // Final state back to [k][v] (coalesced over v).
    if (ok && warp_wait(bar, bar.s_full, (ncl - 1) & 1)) {
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
    // Two warps per TMEM lane quadrant: warp (12 + q + 4 oh) owns value column v = 32 q + lane
    // of the head and tokens [32 oh, 32 oh + 32) of each chunk. Its 32 O^T values are read from
    // TMEM once; the sums of squares over v are reduced across the warp by shuffles and across
    // the four quadrants through shared memory. The 32 gate inputs are loaded before O is waited
    // for, and the per-token arithmetic is branch-free (one warp-uniform bound check per group
    // of eight tokens).
    const unsigned q = warp & 3, oh = (warp - 12) >> 2, v = 32 * q + lane;
    const uint32_t trow = tmem + ((32u * q) << 16);
    float* red = reinterpret_cast<float*>(smem + kOffRed);
    const float nw = a.norm_w[v];
    const float* zh = a.z + h * kDim + v;
    float* out_v = a.out + h * kDim + v;
    constexpr int kG = 8, kT = 32;
    for (unsigned c = 0; c < ncl; ++c) {
      const unsigned b = c & 1, t0 = (c0 + c) * kC + kT * oh;
      const uint32_t ocol = trow + kColO + kT * oh;
      // Tokens past the end read the last token's gate (their outputs are not stored).
      float zr[kT];
#pragma unroll
      for (int i = 0; i < kT; ++i)
        zr[i] = zh[size_t(min(t0 + unsigned(i), a.n - 1)) * a.zab_stride];
      if (!warp_wait(bar, bar.o_full, c & 1))
        break;
      dev::tc_fence_after();
      uint32_t x[kT];
      dev::tmem_ld32(ocol, x);
      dev::tmem_wait_ld();
      // O is in registers: release the TMEM columns to the next chunk's products now.
      dev::tc_fence_before();
      warp_arrive(bar.o_free);
      float* rb = red + b * 4 * kC;
      {
        float s2[kT];
#pragma unroll
        for (int e = 0; e < kT; ++e)
          s2[e] = __uint_as_float(x[e]) * __uint_as_float(x[e]);
        // Reduce-scatter over the warp: lane l ends with token kT oh + l.
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
        rb[q * kC + kT * oh + lane] = s2[0];
      }
      // Exchange through an mbarrier (bounded wait), so a warp that gave up cannot strand the
      // others. Buffer b is rewritten only after every warp has passed the next chunk's wait,
      // i.e. has finished reading it.
      warp_arrive(bar.red_ready[b]);
      if (!warp_wait(bar, bar.red_ready[b], (c >> 1) & 1))
        break;
      const unsigned ti = kT * oh + lane;
      const float r_own = rsqrtf((rb[ti] + rb[kC + ti] + rb[2 * kC + ti] + rb[3 * kC + ti]) *
                                     (1.0f / kDim) + a.eps);
#pragma unroll
      for (int g = 0; g < kT / kG; ++g) {
        float y[kG];
#pragma unroll
        for (int e = 0; e < kG; ++e) {
          const int i = kG * g + e;
          const float r = __shfl_sync(0xffffffffu, r_own, i);
          y[e] = __uint_as_float(x[i]) * r * nw * silu_fast(zr[i]);
        }
        float* dst = out_v + size_t(t0 + kG * g) * kVHeads * kDim;
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
