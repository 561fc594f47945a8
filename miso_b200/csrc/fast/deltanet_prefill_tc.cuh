#pragma once

// Gated DeltaNet prefill (chunked gated delta rule, chunk 64) on the 5th-generation tensor cores:
// the fast path behind miso_deltanet_prefill_tc(). Same inputs, outputs and conv / state
// conventions as the n-token recurrence deltanet_seq (reference kernels/deltanet_step.hpp:146-273;
// chunk algebra of kernels/deltanet_chunk.hpp:3-9).
//
// Per V head h (K head kh = h % 16) and chunk of C = 64 tokens with in-chunk cumulative log decay
// g_i = sum_{t <= i} log(alpha_t) and g_l = g_63:
//   L    = strictly_lower(beta_i e^(g_i - g_j) k_i . k_j),   T = (I + L)^-1   (UT transform)
//   W    = T diag(beta e^g) K,   U = T diag(beta) V                           (WY form)
//   X    = W S,  delta = U - X                     (the delta-rule corrections of the chunk)
//   O    = Qg S + Aqk delta,   Qg = diag(e^g) Q,   Aqk = lower_incl(e^(g_i - g_j) q_i . k_j)
//   S   <- e^(g_l) S + Ks^T delta,   Ks = diag(e^(g_l - g)) K
// and out = O * rsqrt(mean(O^2) + eps) * norm_w * SiLU(z) per token and head.
//
// Three kernels. front_kernel does everything that does not depend on the state, for all chunks
// at once (one CTA per (chunk, K head), both V heads of the K head); chain_kernel runs the state
// recurrence, one CTA per V head, over per-chunk records that front_kernel wrote; gate_kernel
// finishes the outputs:
//   front_kernel  4-tap causal conv + SiLU of the chunk's q / k / v channels straight from the
//                 projection rows, L2 norms, beta and the decays; [K; Q] K^T on tcgen05 (fp16 high
//                 + low operands); L and Aqk; T by a blocked inverse (16 x 16 diagonal blocks, then
//                 the off-diagonal blocks by distance); W = [Tw_0; Tw_1] K and U = Tu V (both V
//                 heads; U from high + low operands); the record of each V head.
//   chain_kernel  per chunk, with the state transposed (S^T, lane = v) as an fp32 TMEM
//                 accumulator and its fp16 high and low parts as TMEM A operands:
//                   [X | O] = S_hi [W; Qg_hi]^T                  (one N = 128 product)
//                   O += S_hi Qg_lo^T + S_lo Qg_hi^T
//                   delta = U - X   (fp16 high + low, into TMEM)
//                   S  += delta_hi Ks_hi + delta_lo Ks_hi + delta_hi Ks_lo
//                   O  += delta_hi Aqk_hi + delta_lo Aqk_hi + delta_hi Aqk_lo
//                 O (double-buffered in TMEM, so the next chunk's products do not wait for it to
//                 be read out), the pre-norm outputs, goes to `out`.
//   gate_kernel   the gated RMS norm of every (token, V head) row, in place (fully parallel).
//
// Precision: every MMA accumulates in fp32 and the state stays fp32. The products that reach the
// outputs or the state through cancelling sums use two-term fp16 operands (hi + lo): the q . k and
// k . k products, U, the output product Qg S, Aqk delta and the state update Ks^T delta. W and the
// state copy in W S are plain fp16 (their rounding is damped by the recurrence). A numpy emulation
// of these rounding points against the fp64 recurrence gives max |error| ~7e-4 of the outputs at
// 32768 tokens (the plain-fp16 variants: 2e-3 to 6e-3), relative L2 ~1e-5.
//
// Records (one per V head and chunk, written by front_kernel, read once by chain_kernel):
//   qgh, qgl [64 i][128 k] fp16    Qg high and low parts
//   w        [64 j][128 k] fp16    W
//   u        [64 j][128 v] fp32    U
//   bh, bl   [192][64 j]   fp16    rows 0..127: Ks^T (row k); rows 128..191: Aqk (row i); high, low
//   egl      fp32                  e^(g_l)
//
// Every mbarrier wait is bounded; on a timeout the block records MISO_STATUS_TIMEOUT (site 0x30
// chain, 0x31 front), stops issuing, drains what it issued and frees its TMEM before exiting.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../common/device.cuh"
#include "../common/tcgen05.cuh"

namespace miso::fast::dnpf {

constexpr int kKHeads = 16, kVHeads = 32, kDim = 128, kC = 64;
constexpr int kQkCh = kKHeads * kDim;            // 2048 q (or k) channels
constexpr int kVCh0 = 2 * kQkCh;                 // first v channel
constexpr uint32_t kBox = 64 * 64 * 2;           // one [64 rows][64] fp16 box: 8 KB

__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(__expf(x)); }

__device__ __forceinline__ uint32_t h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// fp16 pair of two fp32 values and the pair of their remainders (x = hi + lo).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 hv = __floats2half2_rn(x0, x1);
  const float2 f = __half22float2(hv);
  hi = *reinterpret_cast<const uint32_t*>(&hv);
  lo = h2(x0 - f.x, x1 - f.y);
}

__device__ __forceinline__ float2 unpack(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// 4-tap causal conv + SiLU of four channels: taps 0..2 on the three previous inputs (oldest
// first), tap 3 on the current one (kernels/deltanet_step.hpp:50-61).
__device__ __forceinline__ void conv4(const float4 (&w)[4], const float4& a, const float4& b,
                                      const float4& c, const float4& x, float (&y)[4]) {
  y[0] = silu(w[0].x * a.x + w[0].y * b.x + w[0].z * c.x + w[0].w * x.x);
  y[1] = silu(w[1].x * a.y + w[1].y * b.y + w[1].z * c.y + w[1].w * x.y);
  y[2] = silu(w[2].x * a.z + w[2].y * b.z + w[2].z * c.z + w[2].w * x.z);
  y[3] = silu(w[3].x * a.w + w[3].y * b.w + w[3].z * c.w + w[3].w * x.w);
}

// ===================================================================================== records

struct Records {
  __half* qgh;  // [32][nc][64][128]
  __half* qgl;
  __half* w;    // [32][nc][64][128]
  float* u;     // [32][nc][64][128]
  __half* bh;   // [32][nc][192][64]
  __half* bl;
  float* egl;   // [32][nc]
};

__device__ __forceinline__ size_t rec_row(unsigned h, unsigned c, unsigned nc, unsigned rows) {
  return (size_t(h) * nc + c) * rows;
}

// =============================================================================== front_kernel

struct FrontArgs {
  const float* qkv;      // [n][qkv_stride]: q 2048 | k 2048 | v 4096
  const float* a;        // a[t * zab_stride + h]
  const float* b;
  const float* conv_w;   // [8192][4]
  const float* conv_in;  // [8192][3] oldest first
  float* conv_out;
  const float* ssm_a;
  const float* dt_bias;
  Records rec;
  unsigned n, nc, qkv_stride, zab_stride;
  unsigned c0;     // chunk of blockIdx.x = 0 (the launch covers chunks [c0, c0 + gridDim.x))
  unsigned ahead;  // CTAs resident at a time: the unit `ahead` places later is prefetched
  unsigned per;    // chunks per launch when the sequence is covered by consecutive launches
};

constexpr int kFrontThreads = 512;  // 16 warps: 4 tokens each in the convs
constexpr int kLRow = 68;  // fp32 row stride of L (16-byte aligned rows)
// Shared memory (1024-byte aligned base):
//   [0, 64K)      [K; Q] tiles, high parts then low parts: part p, 64-dim slab s at 32K p + 16K s,
//                 K rows 0-63 then Q rows 64-127, 128-byte swizzled ([128 rows][64] fp16)
//   [64K, 128K)   V tiles of both V heads: head hh, part p, slab s at 64K + 8K (4 hh + 2 p + s)
//                 ([64 rows j][64 v] fp16, swizzled; the MN-major B operand of U)
//   [128K, +34K)  L fp32 [2][64][68]
//   then          T fp32 [2][64][68]
//   then          per-head vectors g, beta, e^g, e^(g_l - g), beta e^g [2][64] each
// After the solve the A operands of W and U reuse dead space: Tw at 32K (the low [K; Q] slab 0),
// Tu high at 48K, Tu low at 128K (over L).
// Until the convs have read them, the raw input rows (TMA boxes of [67 rows][128 channels] fp32:
// the chunk's rows and the three before it) occupy [64K, +4 boxes): q, k, then the two v groups
// (dead space then: the V tiles, L and T are written after the convs).
constexpr uint32_t kFOffKQ = 0, kFOffV = 64 * 1024, kFOffL = 128 * 1024;
constexpr int kTRow = 68;  // fp32 row stride of T (rows 64 floats apart would share banks)
constexpr uint32_t kFOffT = kFOffL + 2 * kC * kLRow * 4;
constexpr uint32_t kRawBox = 67 * kDim * 4;  // 34304 bytes
constexpr uint32_t kFOffRaw = 64 * 1024;
constexpr uint32_t kFOffVec = kFOffRaw + 4 * kRawBox;
static_assert(kFOffVec >= kFOffT + 2 * kC * kTRow * 4, "the vectors follow T");
constexpr uint32_t kFOffBar = kFOffVec + 5 * 2 * kC * 4;
constexpr size_t kFrontSmemBytes = kFOffBar + 64;
constexpr uint32_t kFOffTw = 32 * 1024, kFOffTuh = 48 * 1024, kFOffTul = kFOffL;
static_assert(kFrontSmemBytes <= 232448, "fits the opt-in shared memory");
static_assert(2 * kBox <= 2 * kC * kLRow * 4, "Tu low fits in the L area");
// TMEM columns: [K; Q] K^T (64), W (128), U of V head 0 (128), U of V head 1 (128).
constexpr uint32_t kFColKK = 0, kFColW = 64, kFColU0 = 192, kFColU1 = 320;

// Byte offset of channel `ch` (0..127) of row `row` in a [rows][64]-wide swizzled tile pair
// (slab = ch / 64 at `slab_bytes` apart).
__device__ __forceinline__ uint32_t tile_off(uint32_t row, uint32_t ch, uint32_t slab_bytes) {
  return (ch / 64) * slab_bytes + dev::swz128(row, (ch % 64) / 8) + (ch % 8) * 2;
}

// Staging tiles for the record stores: a row of `cpr` 16-byte chunks (cpr a multiple of 8), chunk c
// of row r placed at (c & ~7) | ((c ^ r) & 7), so that row-per-thread writes (lanes on
// consecutive rows) spread over all banks. copy_out() then writes the tile to global memory with
// consecutive lanes on consecutive chunks (512 contiguous bytes per warp store).
__device__ __forceinline__ uint32_t stage_off(uint32_t r, uint32_t c, uint32_t cpr) {
  return (r * cpr + ((c & ~7u) | ((c ^ r) & 7u))) * 16;
}

// Copies `rows` x `cpr` chunks from a staging tile to the contiguous global block dst.
__device__ __forceinline__ void copy_out(const uint8_t* tile, void* dst, uint32_t rows,
                                         uint32_t cpr, unsigned tid, unsigned nthreads) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (uint32_t u = tid; u < rows * cpr; u += nthreads) {
    const uint32_t r = u / cpr, c = u % cpr;
    d[u] = *reinterpret_cast<const uint4*>(tile + stage_off(r, c, cpr));
  }
}

// Off-diagonal blocks of T = (I + L)^-1 (16 x 16 blocks, a > b): T_ab = -T_aa P_ab with
// P_ab = sum_{m=b}^{a-1} L_am T_mb. Thread (row r, column quarter cq) of a block forms
// P_ab[r][4 cq, +4) from its own row of L and broadcast rows of T (phase 1, into P), then
// T_ab[r][4 cq, +4) from its row of T_aa and broadcast rows of P (phase 2). T_aa is lower
// triangular with zeros above the diagonal, so both sums run over all 16 terms.
__device__ __forceinline__ void offdiag_p(const float* L, const float* T, float* P, int a, int b,
                                          int r, int cq) {
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int m = b; m < a; ++m) {
    const float* lr = L + (16 * a + r) * kLRow + 16 * m;
    const float* tc = T + (16 * m) * kTRow + 16 * b + 4 * cq;
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const float4 l4 = *reinterpret_cast<const float4*>(lr + 4 * s4);
      const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float4 t4 = *reinterpret_cast<const float4*>(tc + (4 * s4 + e) * kTRow);
        acc.x += lv[e] * t4.x, acc.y += lv[e] * t4.y, acc.z += lv[e] * t4.z, acc.w += lv[e] * t4.w;
      }
    }
  }
  *reinterpret_cast<float4*>(P + r * 16 + 4 * cq) = acc;
}

__device__ __forceinline__ void offdiag_t(float* T, const float* P, int a, int b, int r, int cq) {
  const float* tr = T + (16 * a + r) * kTRow + 16 * a;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int s4 = 0; s4 < 4; ++s4) {
    const float4 t4 = *reinterpret_cast<const float4*>(tr + 4 * s4);
    const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float4 p4 = *reinterpret_cast<const float4*>(P + (4 * s4 + e) * 16 + 4 * cq);
      acc.x += tv[e] * p4.x, acc.y += tv[e] * p4.y, acc.z += tv[e] * p4.z, acc.w += tv[e] * p4.w;
    }
  }
  *reinterpret_cast<float4*>(T + (16 * a + r) * kTRow + 16 * b + 4 * cq) =
      make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
}

// L2 prefetch of a 2-D box (no data lands in shared memory).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__global__ void __launch_bounds__(kFrontThreads, 1)
    front_kernel(const __grid_constant__ CUtensorMap qkvmap, FrontArgs a) {
  constexpr int kTok = kC / (kFrontThreads / 32);  // tokens per warp in the convs
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((dev::smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0)
      dev::set_status(dev::kStatusTimeout, 0x31);
    return;
  }
  const unsigned c = a.c0 + blockIdx.x, kh = blockIdx.y, tid = threadIdx.x, warp = tid / 32,
                 lane = tid % 32;
  const unsigned nc = a.nc;
  const uint32_t sbase = dev::smem_u32(smem);
  float* Ls = reinterpret_cast<float*>(smem + kFOffL);
  float* Ts = reinterpret_cast<float*>(smem + kFOffT);
  float* gs = reinterpret_cast<float*>(smem + kFOffVec);  // [2][64]
  float* bs = gs + 2 * kC;                                // beta
  float* egs = bs + 2 * kC;                               // e^g
  float* egls = egs + 2 * kC;                             // e^(g_l - g)
  float* fws = egls + 2 * kC;                             // beta e^g
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kFOffBar);  // KK^T, W / U, raw q k, raw v
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  int* fail = reinterpret_cast<int*>(bars + 5);

  if (tid == 0) {
    for (int i = 0; i < 4; ++i)
      dev::mbar_init(dev::smem_u32(&bars[i]), 1);
    *fail = 0;
    dev::mbar_init_fence();
    // The chunk's input rows (and the three before it; rows before the sequence read as zeros
    // and are replaced by the conv history) of the unit's q and k channels, then of its two v
    // channel groups, into shared memory.
    const int y0 = int(c * kC) - 3;
    const uint32_t rq = dev::smem_u32(&bars[2]), rv = dev::smem_u32(&bars[3]);
    dev::mbar_arrive_expect_tx(rq, 2 * kRawBox);
    dev::tma_load_2d(sbase + kFOffRaw, &qkvmap, int(kh * kDim), y0, rq);
    dev::tma_load_2d(sbase + kFOffRaw + kRawBox, &qkvmap, int(kQkCh + kh * kDim), y0, rq);
    dev::mbar_arrive_expect_tx(rv, 2 * kRawBox);
    dev::tma_load_2d(sbase + kFOffRaw + 2 * kRawBox, &qkvmap, int(kVCh0 + kh * kDim), y0, rv);
    dev::tma_load_2d(sbase + kFOffRaw + 3 * kRawBox, &qkvmap,
                     int(kVCh0 + (kh + kKHeads) * kDim), y0, rv);
  }
  // Warps 0 and 1: the a and b inputs of V head kh + 16 warp for the chunk's tokens 2 lane, +1,
  // and the head's ssm_a and dt_bias, loaded now so that their latency overlaps the set-up.
  float av[2] = {0.0f, 0.0f}, bv[2] = {0.0f, 0.0f}, sa_h = 0.0f, dt_h = 0.0f;
  if (warp < 2) {
    const unsigned h = kh + kKHeads * warp;
    sa_h = a.ssm_a[h];
    dt_h = a.dt_bias[h];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const unsigned t = c * kC + 2 * lane + e;
      if (t < a.n) {
        av[e] = a.a[size_t(t) * a.zab_stride + h];
        bv[e] = a.b[size_t(t) * a.zab_stride + h];
      }
    }
  }
  if (warp == 0) {
    dev::tmem_alloc(dev::smem_u32(tmem_slot), 512);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const unsigned t_first = c * kC + kTok * warp;  // warp's first token

  // ---- conv of four channels per lane for the warp's kTok tokens: y[i][e] -------------------
  // Channels ch .. ch + 3 (ch = group base + 4 lane) from the raw box at `raw` (row r = token
  // c * 64 - 3 + r; rows before the sequence come from the conv history instead), with the
  // channels' conv weights w (loaded ahead by load_w).
  auto load_w = [&](unsigned ch, float4 (&w)[4]) {
    const float4* w4 = reinterpret_cast<const float4*>(a.conv_w + 4 * size_t(ch));
#pragma unroll
    for (int e = 0; e < 4; ++e)
      w[e] = w4[e];
  };
  auto conv_rows = [&](uint32_t raw, unsigned ch, const float4 (&w)[4], float (&y)[kTok][4]) {
    const uint8_t* rows = smem + raw + (kTok * warp) * (kDim * 4) + 16 * lane;
    float4 h[3];
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      const int tt = int(t_first) - 3 + s;
      if (tt >= 0) {
        h[s] = *reinterpret_cast<const float4*>(rows + s * (kDim * 4));
      } else {
        const int slot = tt + 3;
        h[s] = make_float4(a.conv_in[3 * ch + slot], a.conv_in[3 * (ch + 1) + slot],
                           a.conv_in[3 * (ch + 2) + slot], a.conv_in[3 * (ch + 3) + slot]);
      }
    }
    float4 xs[kTok];
#pragma unroll
    for (int i = 0; i < kTok; ++i)
      xs[i] = *reinterpret_cast<const float4*>(rows + (3 + i) * (kDim * 4));
#pragma unroll
    for (int i = 0; i < kTok; ++i) {
      conv4(w, h[0], h[1], h[2], xs[i], y[i]);
      h[0] = h[1], h[1] = h[2], h[2] = xs[i];
      if (t_first + i >= a.n)
        y[i][0] = y[i][1] = y[i][2] = y[i][3] = 0.0f;
    }
  };
  // Four consecutive fp32 values of a row as fp16 high / low parts into a swizzled tile pair.
  auto put4 = [&](uint32_t tile, uint32_t row, uint32_t ch, uint32_t slab_bytes,
                  const float (&y)[4], uint32_t lo_tile) {
    uint32_t hi0, lo0, hi1, lo1;
    split2(y[0], y[1], hi0, lo0);
    split2(y[2], y[3], hi1, lo1);
    const uint32_t off = tile_off(row, ch, slab_bytes);
    *reinterpret_cast<uint2*>(smem + tile + off) = make_uint2(hi0, hi1);
    *reinterpret_cast<uint2*>(smem + lo_tile + off) = make_uint2(lo0, lo1);
  };

  // ---- F1: decays and betas (while the raw rows land); q / k conv, L2 norms -> [K; Q] tiles --
  float4 wq[4], wk[4];  // conv weights of the lane's q and k channels
  load_w(kh * kDim + 4 * lane, wq);
  load_w(kQkCh + kh * kDim + 4 * lane, wk);
  if (warp < 2) {
    // In-chunk cumulative log decay and beta of V head kh + 16 warp (beta = 0, no decay past n).
    const unsigned hh = warp, h = kh + kKHeads * hh;
    const unsigned t0 = c * kC + 2 * lane;
    float l[2], bt[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const unsigned t = t0 + e;
      if (t < a.n) {
        l[e] = sa_h * softplus(av[e] + dt_h);
        bt[e] = 1.0f / (1.0f + __expf(-bv[e]));
      } else {
        l[e] = 0.0f, bt[e] = 0.0f;
      }
    }
    float incl = l[0] + l[1];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= unsigned(off))
        incl += y;
    }
    const float g0 = incl - l[1], g1 = incl;
    const float gl = __shfl_sync(0xffffffffu, incl, 31);
    const unsigned i0 = hh * kC + 2 * lane;
    gs[i0] = g0, gs[i0 + 1] = g1;
    bs[i0] = bt[0], bs[i0 + 1] = bt[1];
    const float e0 = __expf(g0), e1 = __expf(g1);
    egs[i0] = e0, egs[i0 + 1] = e1;
    egls[i0] = __expf(gl - g0), egls[i0 + 1] = __expf(gl - g1);
    fws[i0] = bt[0] * e0, fws[i0 + 1] = bt[1] * e1;
    if (lane == 0)
      a.rec.egl[size_t(h) * nc + c] = __expf(gl);
  }
  if (!__all_sync(0xffffffffu, dev::mbar_wait(dev::smem_u32(&bars[2]), 0, 0x31)))
    *fail = 1;  // (the conv then reads stale rows; the status word records the timeout)
  {
    const unsigned ch = 4 * lane;  // channels ch .. ch + 3 of the head
    float yq[kTok][4], yk[kTok][4];
    conv_rows(kFOffRaw, kh * kDim + ch, wq, yq);
    conv_rows(kFOffRaw + kRawBox, kQkCh + kh * kDim + ch, wk, yk);
#pragma unroll
    for (int i = 0; i < kTok; ++i) {
      float sq = yq[i][0] * yq[i][0] + yq[i][1] * yq[i][1] + yq[i][2] * yq[i][2] +
                 yq[i][3] * yq[i][3];
      float sk = yk[i][0] * yk[i][0] + yk[i][1] * yk[i][1] + yk[i][2] * yk[i][2] +
                 yk[i][3] * yk[i][3];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, off);
        sk += __shfl_xor_sync(0xffffffffu, sk, off);
      }
      const float rq = rsqrtf(sq + 1e-6f) * rsqrtf(static_cast<float>(kDim));
      const float rk = rsqrtf(sk + 1e-6f);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        yq[i][e] *= rq, yk[i][e] *= rk;
      const unsigned row = kTok * warp + i;
      put4(kFOffKQ, row, ch, 16 * 1024, yk[i], kFOffKQ + 32 * 1024);
      put4(kFOffKQ, row + kC, ch, 16 * 1024, yq[i], kFOffKQ + 32 * 1024);
    }
  }
  dev::fence_proxy_async_smem();
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();

  // ---- F2: [K; Q] K^T = A_hi B_hi + A_hi B_lo + A_lo B_hi (B = the K rows of A) --------------
  if (tid == 0) {
    const uint32_t idesc = dev::idesc_f16_f32(128, 64, 0, 0);
    const uint64_t hi = dev::sdesc_sw128(sbase + kFOffKQ, 16, 1024);
    const uint64_t lo = dev::sdesc_sw128(sbase + kFOffKQ + 32 * 1024, 16, 1024);
    const uint64_t pa[3] = {hi, hi, lo}, pb[3] = {hi, lo, hi};
#pragma unroll
    for (int t = 0; t < 3; ++t)
#pragma unroll
      for (int ks = 0; ks < kDim / 16; ++ks) {
        const uint64_t off = uint64_t(((ks >> 2) * 16 * 1024 + (ks & 3) * 32) >> 4);
        dev::tc_mma_f16_ss(tmem + kFColKK, pa[t] + off, pb[t] + off, idesc, (t | ks) != 0);
      }
    dev::tc_commit(dev::smem_u32(&bars[0]));
  }

  // ---- F3 (while the MMA runs): v conv of both V heads -> V tiles ----------------------------
  // (The V tiles overlap the raw q / k rows, which every warp has read before the F1 barrier.)
  if (!__all_sync(0xffffffffu, dev::mbar_wait(dev::smem_u32(&bars[3]), 0, 0x31)))
    *fail = 1;
#pragma unroll 1
  for (unsigned hh = 0; hh < 2; ++hh) {
    const unsigned ch = 4 * lane;
    float yv[kTok][4];
    float4 wv[4];
    load_w(kVCh0 + (kh + kKHeads * hh) * kDim + ch, wv);
    conv_rows(kFOffRaw + (2 + hh) * kRawBox, kVCh0 + (kh + kKHeads * hh) * kDim + ch, wv, yv);
    const uint32_t vt = kFOffV + 4 * hh * kBox;
#pragma unroll
    for (int i = 0; i < kTok; ++i)
      put4(vt, kTok * warp + i, ch, kBox, yv[i], vt + 2 * kBox);
  }
  // The final conv history (the last three input rows) of this unit's channels.
  if (c == nc - 1) {
    for (unsigned u = tid; u < 4 * kDim * 3; u += kFrontThreads) {
      const unsigned slot = u % 3, cc = u / 3, part = cc / kDim, e = cc % kDim;
      const unsigned ch = part == 0   ? kh * kDim + e
                          : part == 1 ? kQkCh + kh * kDim + e
                                      : kVCh0 + (kh + kKHeads * (part - 2)) * kDim + e;
      const int tt = int(a.n) - 3 + int(slot);
      a.conv_out[3 * ch + slot] =
          tt >= 0 ? a.qkv[size_t(tt) * a.qkv_stride + ch] : a.conv_in[3 * ch + slot + a.n];
    }
  }

  // ---- F4: L and Aqk from the product -------------------------------------------------------
  __syncthreads();  // every warp is past the v conv: L and T may overwrite the raw v rows
  const bool mma_ok = dev::mbar_wait(dev::smem_u32(&bars[0]), 0, 0x31);
  if (!mma_ok)
    *fail = 1;
  dev::tc_fence_after();
  if (__all_sync(0xffffffffu, mma_ok)) {
    // Warp w: TMEM lanes [32 (w % 4), +32) (product rows), columns [16 (w / 4), +16) (j).
    const unsigned r = 32 * (warp % 4) + lane, jb = 16 * (warp / 4);
    uint32_t x[16];
    dev::tmem_ld16(tmem + ((32u * (warp % 4)) << 16) + kFColKK + jb, x);
    dev::tmem_wait_ld();
    if (r < kC) {  // k_r . k_j
      const unsigned i = r;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float gi = gs[hh * kC + i], bi = bs[hh * kC + i];
        float* row = Ls + (hh * kC + i) * kLRow + jb;
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = int(jb) + 4 * j4 + e;
            v[e] = j < int(i) ? bi * __expf(gi - gs[hh * kC + j]) * __uint_as_float(x[4 * j4 + e])
                              : 0.0f;
          }
          *reinterpret_cast<float4*>(row + 4 * j4) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
    } else {  // q_i . k_j -> Aqk (high, low) staged in the T area: [hh][part][64 i][64 j]
      const unsigned i = r - kC;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float gi = gs[hh * kC + i];
        uint8_t* sh = smem + kFOffT + (2 * hh) * kBox;
        uint8_t* sl = sh + kBox;
#pragma unroll
        for (int q8 = 0; q8 < 2; ++q8) {
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j0 = int(jb) + 8 * q8 + 2 * e;
            const float v0 = j0 <= int(i) ? __expf(gi - gs[hh * kC + j0]) *
                                                __uint_as_float(x[8 * q8 + 2 * e])
                                          : 0.0f;
            const float v1 = j0 + 1 <= int(i) ? __expf(gi - gs[hh * kC + j0 + 1]) *
                                                    __uint_as_float(x[8 * q8 + 2 * e + 1])
                                              : 0.0f;
            split2(v0, v1, hi[e], lo[e]);
          }
          const uint32_t off = stage_off(i, jb / 8 + q8, 8);
          *reinterpret_cast<uint4*>(sh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(sl + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
      }
    }
  }
  dev::tc_fence_before();
  __syncthreads();
  if (!*reinterpret_cast<volatile int*>(fail)) {
#pragma unroll 1
    for (int part = 0; part < 4; ++part) {  // (hh, high / low): rows 128..191 of bh / bl
      const unsigned hh = part / 2, h = kh + kKHeads * hh;
      __half* dst = ((part & 1) ? a.rec.bl : a.rec.bh) + (rec_row(h, c, nc, 192) + 128) * kC;
      copy_out(smem + kFOffT + part * kBox, dst, kC, 8, tid, kFrontThreads);
    }
  }
  dev::tc_fence_before();
  __syncthreads();

  const bool ok = !*reinterpret_cast<volatile int*>(fail);
  if (ok) {
    // ---- F5: Qg = Q e^g and Ks^T = (K e^(g_l - g))^T, high and low parts ---------------------
    // Qg: 16-byte unit u = (row i = u / 16, dims 8 (u % 16) .. + 7), consecutive lanes on
    // consecutive units, so each warp store is 512 contiguous bytes.
#pragma unroll 1
    for (unsigned u = tid; u < kC * 16; u += kFrontThreads) {
      const unsigned i = u / 16, k0 = 8 * (u % 16);
      const uint32_t off = tile_off(kC + i, k0, 16 * 1024);
      const uint4 hi = *reinterpret_cast<const uint4*>(smem + kFOffKQ + off);
      const uint4 lo = *reinterpret_cast<const uint4*>(smem + kFOffKQ + 32 * 1024 + off);
      const uint32_t hw[4] = {hi.x, hi.y, hi.z, hi.w}, lw[4] = {lo.x, lo.y, lo.z, lo.w};
      float q[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fh = unpack(hw[e]), fl = unpack(lw[e]);
        q[2 * e] = fh.x + fl.x;
        q[2 * e + 1] = fh.y + fl.y;
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const unsigned h = kh + kKHeads * hh;
        const float f = egs[hh * kC + i];
        uint32_t oh[4], ol[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          split2(q[2 * e] * f, q[2 * e + 1] * f, oh[e], ol[e]);
        const size_t ro = (rec_row(h, c, nc, kC) + i) * kDim + k0;
        *reinterpret_cast<uint4*>(a.rec.qgh + ro) = make_uint4(oh[0], oh[1], oh[2], oh[3]);
        *reinterpret_cast<uint4*>(a.rec.qgl + ro) = make_uint4(ol[0], ol[1], ol[2], ol[3]);
      }
    }
    // Ks^T, one V head at a time through the T area: thread (row k = tid % 128, j quarter
    // tid / 128) writes its 16 values into the staging tile, then the tile is copied out.
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
      const unsigned h = kh + kKHeads * hh, k = tid % kDim, j0 = 16 * (tid / kDim);
      uint8_t* sh = smem + kFOffT;
      uint8_t* sl = sh + 2 * kBox;
#pragma unroll
      for (int q8 = 0; q8 < 2; ++q8) {
        uint32_t oh[4], ol[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v[2];
#pragma unroll
          for (int f = 0; f < 2; ++f) {
            const unsigned j = j0 + 8 * q8 + 2 * e + f;
            const uint32_t off = tile_off(j, k, 16 * 1024);
            const float x =
                __half2float(*reinterpret_cast<const __half*>(smem + kFOffKQ + off)) +
                __half2float(*reinterpret_cast<const __half*>(smem + kFOffKQ + 32 * 1024 + off));
            v[f] = x * egls[hh * kC + j];
          }
          split2(v[0], v[1], oh[e], ol[e]);
        }
        const uint32_t off = stage_off(k, j0 / 8 + q8, 8);
        *reinterpret_cast<uint4*>(sh + off) = make_uint4(oh[0], oh[1], oh[2], oh[3]);
        *reinterpret_cast<uint4*>(sl + off) = make_uint4(ol[0], ol[1], ol[2], ol[3]);
      }
      __syncthreads();
      copy_out(sh, a.rec.bh + rec_row(h, c, nc, 192) * kC, kDim, 8, tid, kFrontThreads);
      copy_out(sl, a.rec.bl + rec_row(h, c, nc, 192) * kC, kDim, 8, tid, kFrontThreads);
      __syncthreads();
    }

    // Bring the input rows of the unit that will run `ahead` CTAs later (the next wave, roughly)
    // into L2 while this one finishes: issued about two thirds into the CTA, so that the rows are
    // still in L2 when that unit starts (earlier, the records and the concurrent chain's traffic
    // evicted them).
    // Units run in launch order (chunk fastest, then K head), launch after launch: the unit
    // `ahead` places later may belong to the next launch (chunks [c0 + gridDim.x, + per)).
    if (tid == 0) {
      unsigned nid = blockIdx.y * gridDim.x + blockIdx.x + a.ahead, c2 = nc, kh2 = 0;
      if (nid < gridDim.x * gridDim.y) {
        c2 = a.c0 + nid % gridDim.x, kh2 = nid / gridDim.x;
      } else if (a.c0 + gridDim.x < nc) {
        const unsigned c1 = a.c0 + gridDim.x, cnt = nc - c1 < a.per ? nc - c1 : a.per;
        nid -= gridDim.x * gridDim.y;
        if (nid < cnt * kKHeads)
          c2 = c1 + nid % cnt, kh2 = nid / cnt;
      }
      if (c2 < nc) {
        const int y0 = int(c2 * kC) - 3;
        tma_prefetch_2d(&qkvmap, int(kh2 * kDim), y0);
        tma_prefetch_2d(&qkvmap, int(kQkCh + kh2 * kDim), y0);
        tma_prefetch_2d(&qkvmap, int(kVCh0 + kh2 * kDim), y0);
        tma_prefetch_2d(&qkvmap, int(kVCh0 + (kh2 + kKHeads) * kDim), y0);
      }
    }

    // ---- F6: T = (I + L)^-1 of both heads, blocked by 16 ------------------------------------
    // Diagonal blocks by forward substitution: thread (hh, block a, column q).
    if (tid < 128) {
      const unsigned hh = tid / 64, ab = (tid / 16) % 4, q = tid % 16;
      const float* L = Ls + hh * kC * kLRow;
      float* T = Ts + hh * kC * kTRow;
      const int i0 = 16 * int(ab);
      float t[16];
#pragma unroll
      for (int r = 0; r < 16; ++r)
        t[r] = r == int(q) ? 1.0f : 0.0f;
#pragma unroll
      for (int r = 1; r < 16; ++r) {
        const float* lr = L + (i0 + r) * kLRow + i0;
#pragma unroll
        for (int s = 0; s < r; ++s)
          t[r] -= lr[s] * t[s];
      }
#pragma unroll
      for (int r = 0; r < 16; ++r)
        T[(i0 + r) * kTRow + i0 + int(q)] = t[r];
    }
    __syncthreads();
    // Off-diagonal blocks by distance d = a - b: 3, 2 and 1 blocks per head; thread (hh, block,
    // row r, column quarter cq), whole warps active or idle. P goes through the Q rows of the
    // high [K; Q] slab 0 (dead once Qg has been formed): [hh][block][16][16] fp32.
    float* Ps = reinterpret_cast<float*>(smem + kFOffKQ + 8 * 1024);
#pragma unroll 1
    for (int d = 1; d < 4; ++d) {
      const int nb = 4 - d;
      const int u = int(tid), cq = u % 4, r = (u / 4) % 16, blk = (u / 64) % nb,
                hh = u / (64 * nb);
      const bool act = tid < unsigned(2 * nb * 64);
      float* P = Ps + (hh * nb + blk) * 256;
      if (act)
        offdiag_p(Ls + hh * kC * kLRow, Ts + hh * kC * kTRow, P, blk + d, blk, r, cq);
      __syncthreads();
      if (act)
        offdiag_t(Ts + hh * kC * kTRow, P, blk + d, blk, r, cq);
      __syncthreads();
    }

    // ---- F7: A operands of W and U: Tw = T diag(beta e^g) (fp16), Tu = T diag(beta) (hi, lo);
    // rows (hh, i) of [128 rows][64 j] swizzled tiles, 16-byte chunk u: row u / 8, j 8 (u % 8).
#pragma unroll 2
    for (unsigned u = tid; u < 2 * kC * 8; u += kFrontThreads) {
      const unsigned cc = u % 8, r = u / 8, hh = r / kC, i = r % kC;
      const float* t = Ts + r * kTRow + 8 * cc;
      uint32_t w4[4], uh[4], ul[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j0 = int(8 * cc) + 2 * e;
        const float t0 = j0 <= int(i) ? t[2 * e] : 0.0f;
        const float t1 = j0 + 1 <= int(i) ? t[2 * e + 1] : 0.0f;
        w4[e] = h2(t0 * fws[hh * kC + j0], t1 * fws[hh * kC + j0 + 1]);
        split2(t0 * bs[hh * kC + j0], t1 * bs[hh * kC + j0 + 1], uh[e], ul[e]);
      }
      const uint32_t off = dev::swz128(r, cc);
      *reinterpret_cast<uint4*>(smem + kFOffTw + off) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      *reinterpret_cast<uint4*>(smem + kFOffTuh + off) = make_uint4(uh[0], uh[1], uh[2], uh[3]);
      *reinterpret_cast<uint4*>(smem + kFOffTul + off) = make_uint4(ul[0], ul[1], ul[2], ul[3]);
    }
    dev::fence_proxy_async_smem();
  }
  dev::tc_fence_before();
  __syncthreads();

  // ---- F8: W = [Tw_0; Tw_1] K (both heads, M = 128) and U = [Tu_0; Tu_1] V_hh per head (the
  // rows of the other head are discarded), U from Tu_hi V_hi + Tu_hi V_lo + Tu_lo V_hi ----------
  if (tid == 0 && ok) {
    dev::tc_fence_after();
    const uint32_t id_w = dev::idesc_f16_f32(128, 128, 0, 1);  // A K-major, B MN-major
    auto adesc = [&](uint32_t off, int kk) {
      return dev::sdesc_sw128(sbase + off + kk * 32, 16, 1024);
    };
#pragma unroll
    for (int kk = 0; kk < kC / 16; ++kk)
      dev::tc_mma_f16_ss(tmem + kFColW, adesc(kFOffTw, kk),
                         dev::sdesc_sw128(sbase + kFOffKQ + kk * 2048, 16 * 1024, 1024), id_w,
                         kk > 0);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const uint32_t vt = kFOffV + 4 * hh * kBox;
      const uint32_t ta[3] = {kFOffTuh, kFOffTuh, kFOffTul};
      const uint32_t tb[3] = {vt, vt + 2 * kBox, vt};
#pragma unroll
      for (int p = 0; p < 3; ++p)
#pragma unroll
        for (int kk = 0; kk < kC / 16; ++kk)
          dev::tc_mma_f16_ss(tmem + (hh ? kFColU1 : kFColU0), adesc(ta[p], kk),
                             dev::sdesc_sw128(sbase + tb[p] + kk * 2048, kBox, 1024), id_w,
                             (p | kk) != 0);
    }
    dev::tc_commit(dev::smem_u32(&bars[1]));
  }
  __syncthreads();

  // ---- F9: W (fp16) and U (fp32) rows through staging tiles (the [K; Q] and V areas are free
  // once the products are done) to the records --------------------------------------------------
  const bool wu_ok =
      ok && __all_sync(0xffffffffu, dev::mbar_wait(dev::smem_u32(&bars[1]), 0, 0x31));
  if (wu_ok) {
    dev::tc_fence_after();
    const unsigned r = 32 * (warp % 4) + lane, hh = r / kC, i = r % kC;
    const unsigned cb = 32 * (warp / 4);  // this warp's 32 of the 128 columns
    const uint32_t trow = tmem + ((32u * (warp % 4)) << 16);
    uint8_t* ws = smem + kFOffKQ + hh * 16 * 1024;  // [64 rows][16 chunks] fp16
    uint8_t* us = smem + kFOffV + hh * 32 * 1024;   // [64 rows][32 chunks] fp32
    {
      constexpr int part = 0;
      uint32_t x[32];
      dev::tmem_ld32(trow + kFColW + cb + 32 * part, x);
      dev::tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(ws + stage_off(i, (cb + 32 * part) / 8 + q, 16)) = make_uint4(
            h2(__uint_as_float(x[8 * q]), __uint_as_float(x[8 * q + 1])),
            h2(__uint_as_float(x[8 * q + 2]), __uint_as_float(x[8 * q + 3])),
            h2(__uint_as_float(x[8 * q + 4]), __uint_as_float(x[8 * q + 5])),
            h2(__uint_as_float(x[8 * q + 6]), __uint_as_float(x[8 * q + 7])));
      dev::tmem_ld32(trow + (hh ? kFColU1 : kFColU0) + cb + 32 * part, x);
      dev::tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<uint4*>(us + stage_off(i, (cb + 32 * part) / 4 + q, 32)) =
            make_uint4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
    }
  }
  __syncthreads();
  if (wu_ok) {
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
      const unsigned h = kh + kKHeads * hh;
      copy_out(smem + kFOffKQ + hh * 16 * 1024, a.rec.w + rec_row(h, c, nc, kC) * kDim, kC, 16,
               tid, kFrontThreads);
      copy_out(smem + kFOffV + hh * 32 * 1024, a.rec.u + rec_row(h, c, nc, kC) * kDim, kC, 32,
               tid, kFrontThreads);
    }
  }
  dev::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, 512);
  }
  // After a timed-out wait on the raw rows, no copy may still land once the CTA has exited:
  // wait (bounded) for both (a completed phase passes at once).
  if (tid == 0 && *reinterpret_cast<volatile int*>(fail)) {
    dev::mbar_wait(dev::smem_u32(&bars[2]), 0);
    dev::mbar_wait(dev::smem_u32(&bars[3]), 0);
  }
}

// =============================================================================== chain_kernel

struct ChainArgs {
  const float* egl;  // [32][nc] e^(g_l)
  float* state;      // [32][128 k][128 v]: read before chunk c0, written after the last one
  float* out;        // [n][4096]: the pre-norm outputs O (gate_kernel finishes them)
  unsigned n, nc;
  unsigned c0, cnt;  // the launch runs chunks [c0, c0 + cnt)
};

constexpr int kChainThreads = 448;  // warp 0 TMA, warp 1 MMA, 2-9 state, 10-13 output
// Shared memory: the B operands of the [X | O] products, double-buffered (per 64-dim slab, 24 KB:
// rows [W; Qg_hi; Qg_lo] in stage 0 and [Qg_hi; W; Qg_lo] in stage 1, matching the column order
// of the two O buffers), the [Ks^T; Aqk] tiles (high, low; 24 KB each), double-buffered,
// U (fp32, four [64 j][32 v] blocks; single, it is read by the state warps early in each chunk).
constexpr uint32_t kXySlab = 3 * kBox, kXyStage = 2 * kXySlab;  // 24 KB, 48 KB
constexpr uint32_t kBStage = 6 * kBox;                          // [Ks^T; Aqk] high + low: 48 KB
constexpr uint32_t kCOffXy = 0, kCOffB = 2 * kXyStage, kCOffU = kCOffB + 2 * kBStage;
constexpr uint32_t kCOffBar = kCOffU + 32 * 1024;

struct ChainBars {
  uint64_t xy_full[2], xy_empty[2], b_full[2], b_empty[2], u_full, u_empty;
  uint64_t sh_ready, sl_ready, s_scaled, x_full, d_ready, s_full, o_full[2], o_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t kChainSmemBytes = kCOffBar + sizeof(ChainBars);
static_assert(kChainSmemBytes <= 232448, "fits the opt-in shared memory");

// TMEM columns (lane = value row v of the M = 128 tiles): the fp32 state S^T, O^T of odd chunks,
// X^T, O^T of even chunks ([X | O_even] and [O_odd | X] are each one N = 128 accumulator), the
// fp16 state copies (A operands, two k per column), delta^T high and low parts.
constexpr uint32_t kColS = 0, kColO1 = 128, kColX = 192, kColO0 = 256, kColSh = 320,
                   kColSl = 384, kColDh = 448, kColDl = 480;

__device__ __forceinline__ bool aborted(const ChainBars& b) {
  return *reinterpret_cast<const volatile int*>(&b.abort_flag) != 0;
}

__device__ __forceinline__ bool wait_or_abort(ChainBars& b, uint64_t& bar, uint32_t parity) {
  if (aborted(b))
    return false;
  if (!dev::mbar_wait(dev::smem_u32(&bar), parity, 0x30)) {
    b.abort_flag = 1;
    return false;
  }
  return true;
}

// Single-thread bounded wait that polls (mbarrier.test_wait) instead of suspending in try_wait:
// the MMA issuer resumes as soon as the phase completes.
__device__ __forceinline__ bool poll_or_abort(ChainBars& b, uint64_t& bar, uint32_t parity) {
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
__device__ __forceinline__ bool warp_wait(ChainBars& b, uint64_t& bar, uint32_t parity) {
  return __all_sync(0xffffffffu, wait_or_abort(b, bar, parity));
}

__device__ __forceinline__ void warp_arrive(uint64_t& bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0)
    dev::mbar_arrive(dev::smem_u32(&bar));
}

__global__ void __launch_bounds__(kChainThreads, 1)
    chain_kernel(const __grid_constant__ CUtensorMap qghmap,
                 const __grid_constant__ CUtensorMap qglmap,
                 const __grid_constant__ CUtensorMap wmap,
                 const __grid_constant__ CUtensorMap umap,
                 const __grid_constant__ CUtensorMap bhmap,
                 const __grid_constant__ CUtensorMap blmap, ChainArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if ((dev::smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0)
      dev::set_status(dev::kStatusTimeout, 0x30);
    return;
  }
  ChainBars& bar = *reinterpret_cast<ChainBars*>(smem + kCOffBar);
  const unsigned h = blockIdx.x, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const unsigned nc = a.nc, cnt = a.cnt;
  const uint32_t sbase = dev::smem_u32(smem);

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(dev::smem_u32(&bar.xy_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.xy_empty[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.b_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.b_empty[s]), 1);
    }
    dev::mbar_init(dev::smem_u32(&bar.u_full), 1);
    dev::mbar_init(dev::smem_u32(&bar.u_empty), 8);
    dev::mbar_init(dev::smem_u32(&bar.sh_ready), 8);
    dev::mbar_init(dev::smem_u32(&bar.sl_ready), 8);
    dev::mbar_init(dev::smem_u32(&bar.s_scaled), 8);
    dev::mbar_init(dev::smem_u32(&bar.x_full), 1);
    dev::mbar_init(dev::smem_u32(&bar.d_ready), 8);
    dev::mbar_init(dev::smem_u32(&bar.s_full), 1);
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(dev::smem_u32(&bar.o_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.o_free[s]), 4);
    }
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
      dev::tma_prefetch_desc(&qghmap);
      dev::tma_prefetch_desc(&wmap);
      dev::tma_prefetch_desc(&umap);
      dev::tma_prefetch_desc(&bhmap);
      unsigned xy_issued = 0, u_issued = 0, b_issued = 0;
      for (unsigned c = 0; c < cnt; ++c) {  // (c counts the launch's chunks)
        const unsigned s = c & 1;
        const int row64 = int(rec_row(h, a.c0 + c, nc, kC));
        const int row192 = int(rec_row(h, a.c0 + c, nc, 192));
        // [X | O] operands of chunk c (stage s free once chunk c - 2's products are done):
        // rows [W; Qg_hi; Qg_lo] for even chunks, [Qg_hi; W; Qg_lo] for odd ones
        if (c >= 2 && !wait_or_abort(bar, bar.xy_empty[s], ((c >> 1) & 1) ^ 1))
          break;
        const uint32_t xs = sbase + kCOffXy + s * kXyStage, xf = dev::smem_u32(&bar.xy_full[s]);
        dev::mbar_arrive_expect_tx(xf, kXyStage);
        for (int x = 0; x < 2; ++x) {
          dev::tma_load_2d(xs + x * kXySlab + (s ? 0 : kBox), &qghmap, x * 64, row64, xf);
          dev::tma_load_2d(xs + x * kXySlab + 2 * kBox, &qglmap, x * 64, row64, xf);
          dev::tma_load_2d(xs + x * kXySlab + (s ? kBox : 0), &wmap, x * 64, row64, xf);
        }
        xy_issued = c + 1;
        // [Ks^T; Aqk] of chunk c (stage s free once chunk c - 2's updates are done)
        if (c >= 2 && !wait_or_abort(bar, bar.b_empty[s], ((c >> 1) & 1) ^ 1))
          break;
        const uint32_t bs = sbase + kCOffB + s * kBStage, bf = dev::smem_u32(&bar.b_full[s]);
        dev::mbar_arrive_expect_tx(bf, kBStage);
        dev::tma_load_2d(bs, &bhmap, 0, row192, bf);
        dev::tma_load_2d(bs + 3 * kBox, &blmap, 0, row192, bf);
        b_issued = c + 1;
        // U of chunk c (after the state warps have read chunk c - 1's)
        if (c >= 1 && !wait_or_abort(bar, bar.u_empty, (c - 1) & 1))
          break;
        const uint32_t uf = dev::smem_u32(&bar.u_full);
        dev::mbar_arrive_expect_tx(uf, 32 * 1024);
        for (int x = 0; x < 4; ++x)
          dev::tma_load_2d(sbase + kCOffU + x * 8192, &umap, x * 32, row64, uf);
        u_issued = c + 1;
      }
      if (aborted(bar)) {  // let the copies already issued land before the CTA exits (bounded)
        for (unsigned c = xy_issued >= 2 ? xy_issued - 2 : 0; c < xy_issued; ++c)
          dev::mbar_wait(dev::smem_u32(&bar.xy_full[c & 1]), (c >> 1) & 1);
        for (unsigned c = b_issued >= 2 ? b_issued - 2 : 0; c < b_issued; ++c)
          dev::mbar_wait(dev::smem_u32(&bar.b_full[c & 1]), (c >> 1) & 1);
        if (u_issued > 0)
          dev::mbar_wait(dev::smem_u32(&bar.u_full), (u_issued - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------ MMA issue
    // Per chunk c (O buffer b = c % 2), in issue order (the tensor pipe runs them in order):
    //   XY1  [X | O_b] = S_hi [W; Qg_hi]^T     after E0 wrote S_hi, O_b of chunk c - 2 was read
    //   XY2  O_b += S_hi Qg_lo^T + S_lo Qg_hi^T  (the latter after E0 wrote S_lo)
    //   C2   S += D_hi Ks_hi + D_lo Ks_hi + D_hi Ks_lo    after E1 wrote delta, S was scaled
    //   Z    O_b += D_hi A_hi + D_lo A_hi + D_hi A_lo
    if (lane == 0) {
      const uint32_t id_128 = dev::idesc_f16_f32(128, 128, 0, 0);
      const uint32_t id_64 = dev::idesc_f16_f32(128, 64, 0, 0);
      auto kdesc = [](uint32_t addr) { return dev::sdesc_sw128(addr, 16, 1024); };
      bool ok = true;
      for (unsigned c = 0; ok && c < cnt; ++c) {
        const unsigned s = c & 1;
        const uint32_t xs = sbase + kCOffXy + s * kXyStage;
        const uint32_t ocol = s ? kColO1 : kColO0, xycol = s ? kColO1 : kColX;
        const uint32_t qgh_row = s ? 0 : kBox;  // Qg_hi rows in the stage (byte offset in a slab)
        if (!poll_or_abort(bar, bar.xy_full[s], (c >> 1) & 1) ||
            !poll_or_abort(bar, bar.sh_ready, c & 1) ||
            (c >= 2 && !poll_or_abort(bar, bar.o_free[s], ((c >> 1) & 1) ^ 1))) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          dev::tc_mma_f16_ts(tmem + xycol, tmem + kColSh + 8 * ks,
                             kdesc(xs + (ks >> 2) * kXySlab + (ks & 3) * 32), id_128, ks > 0);
        dev::tc_commit(dev::smem_u32(&bar.x_full));
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          dev::tc_mma_f16_ts(tmem + ocol, tmem + kColSh + 8 * ks,
                             kdesc(xs + (ks >> 2) * kXySlab + 2 * kBox + (ks & 3) * 32), id_64, 1);
        if (!poll_or_abort(bar, bar.sl_ready, c & 1)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          dev::tc_mma_f16_ts(tmem + ocol, tmem + kColSl + 8 * ks,
                             kdesc(xs + (ks >> 2) * kXySlab + qgh_row + (ks & 3) * 32), id_64, 1);
        dev::tc_commit(dev::smem_u32(&bar.xy_empty[s]));
        if (!poll_or_abort(bar, bar.b_full[s], (c >> 1) & 1) ||
            !poll_or_abort(bar, bar.d_ready, c & 1) || !poll_or_abort(bar, bar.s_scaled, c & 1)) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const uint32_t bs = sbase + kCOffB + s * kBStage;
        const uint32_t da[3] = {kColDh, kColDl, kColDh};
        const uint32_t bb[3] = {bs, bs, bs + 3 * kBox};
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            dev::tc_mma_f16_ts(tmem + kColS, tmem + da[p] + 8 * kk, kdesc(bb[p] + kk * 32), id_128,
                               1);
        dev::tc_commit(dev::smem_u32(&bar.s_full));
#pragma unroll
        for (int p = 0; p < 3; ++p)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            dev::tc_mma_f16_ts(tmem + ocol, tmem + da[p] + 8 * kk,
                               kdesc(bb[p] + 16 * 1024 + kk * 32), id_64, 1);
        dev::tc_commit(dev::smem_u32(&bar.o_full[s]));
        dev::tc_commit(dev::smem_u32(&bar.b_empty[s]));
      }
      dev::tc_commit(dev::smem_u32(&bar.drain));
      dev::mbar_wait(dev::smem_u32(&bar.drain), 0);
    }
  } else if (warp >= 2 && warp < 10) {
    // ------------------------------------------- state warps: S copies, S decay, delta = U - X
    // Warp w: TMEM lanes [32 q, +32) with q = w % 4 (rows v), S^T columns (k) [64 hc, +64) with
    // hc = (w - 2) / 4, X^T columns (j) [32 hc, +32).
    const unsigned q = warp & 3, hc = (warp - 2) >> 2, v = 32 * q + lane;
    const uint32_t trow = tmem + ((32u * q) << 16);
    const float* S = a.state + size_t(h) * kDim * kDim;
    const float* us = reinterpret_cast<const float*>(smem + kCOffU + q * 8192) + lane;
    bool ok = true;
    for (unsigned c = 0; ok && c < cnt; ++c) {
      const float el = a.egl[size_t(h) * nc + a.c0 + c];
      // E0: the fp16 high copy of S^T first (the A operand the next product waits for), then,
      // reading S^T again, the low copy and S^T *= e^(g_l). 32 columns at a time.
      if (c > 0 && !warp_wait(bar, bar.s_full, (c - 1) & 1)) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
      auto load_s = [&](int half, uint32_t (&x)[32]) {
        if (c == 0) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            x[e] = __float_as_uint(S[size_t(64 * hc + 32 * half + e) * kDim + v]);
        } else {
          dev::tmem_ld32(trow + kColS + 64 * hc + 32 * half, x);
          dev::tmem_wait_ld();
        }
      };
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t x[32], ph[16];
        load_s(half, x);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          ph[e] = h2(__uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]));
        dev::tmem_st16(trow + kColSh + 32 * hc + 16 * half, ph);
      }
      dev::tmem_wait_st();
      dev::tc_fence_before();
      warp_arrive(bar.sh_ready);
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t x[32], pl[16];
        load_s(half, x);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          uint32_t hi;
          split2(__uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]), hi, pl[e]);
        }
        dev::tmem_st16(trow + kColSl + 32 * hc + 16 * half, pl);
#pragma unroll
        for (int e = 0; e < 32; ++e)
          x[e] = __float_as_uint(__uint_as_float(x[e]) * el);
        dev::tmem_st32(trow + kColS + 64 * hc + 32 * half, x);
      }
      dev::tmem_wait_st();
      dev::tc_fence_before();
      warp_arrive(bar.sl_ready);
      warp_arrive(bar.s_scaled);

      // E1: delta^T = U^T - X^T as fp16 high part and remainder.
      if (!warp_wait(bar, bar.x_full, c & 1) || !warp_wait(bar, bar.u_full, c & 1)) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
      uint32_t xx[32];
      dev::tmem_ld32(trow + kColX + 32 * hc, xx);
      dev::tmem_wait_ld();
      uint32_t dh[16], dl[16];
      const float* uj = us + 32 * hc * 32;
#pragma unroll
      for (int e = 0; e < 16; ++e)
        split2(uj[(2 * e) * 32] - __uint_as_float(xx[2 * e]),
               uj[(2 * e + 1) * 32] - __uint_as_float(xx[2 * e + 1]), dh[e], dl[e]);
      warp_arrive(bar.u_empty);
      dev::tmem_st16(trow + kColDh + 16 * hc, dh);
      dev::tmem_st16(trow + kColDl + 16 * hc, dl);
      dev::tmem_wait_st();
      dev::tc_fence_before();
      warp_arrive(bar.d_ready);
    }
    // Final state back to [k][v] (coalesced over v).
    if (ok && warp_wait(bar, bar.s_full, (cnt - 1) & 1)) {
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
  } else if (warp >= 10) {
    // ------------------------------------------------------------ output warps: raw O to out
    // Warp w owns value column v = 32 (w % 4) + lane of the head: per chunk it reads O of the
    // chunk's 64 tokens from TMEM, releases the columns, and stores them into `out`
    // (one 128-byte row segment per token and warp). gate_kernel applies the norm and the gate.
    const unsigned q = warp & 3, v = 32 * q + lane;
    const uint32_t trow = tmem + ((32u * q) << 16);
    float* out_v = a.out + h * kDim + v;
    for (unsigned c = 0; c < cnt; ++c) {
      const unsigned b = c & 1;
      if (!warp_wait(bar, bar.o_full[b], (c >> 1) & 1))
        break;
      dev::tc_fence_after();
      float o[kC];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t x[32];
        dev::tmem_ld32(trow + (b ? kColO1 : kColO0) + 32 * half, x);
        dev::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          o[32 * half + e] = __uint_as_float(x[e]);
      }
      dev::tc_fence_before();
      warp_arrive(bar.o_free[b]);  // O_b is in registers: release it
      const unsigned t0 = (a.c0 + c) * kC;
      float* dst = out_v + size_t(t0) * kVHeads * kDim;
      if (t0 + kC <= a.n) {
#pragma unroll
        for (int e = 0; e < kC; ++e)
          dst[size_t(e) * kVHeads * kDim] = o[e];
      } else {
#pragma unroll
        for (int e = 0; e < kC; ++e)
          if (t0 + e < a.n)
            dst[size_t(e) * kVHeads * kDim] = o[e];
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

// ================================================================================ gate_kernel

// out = O * rsqrt(mean_v(O^2) + eps) * norm_w * SiLU(z) per (token, V head), in place over the
// pre-norm outputs chain_kernel wrote (the gated RMS norm of kernels/deltanet_step.hpp:124-131).
// One warp per (token, head) row of 128 values, four per lane; rows are grid-strided.
struct GateArgs {
  float* out;           // [n][4096]
  const float* z;       // z[t * zab_stride + h * 128 + v]
  const float* norm_w;  // [128]
  unsigned n, zab_stride;
  float eps;
  unsigned t0;          // the launch covers tokens [t0, n)
};

constexpr int kGateThreads = 256;

__global__ void __launch_bounds__(kGateThreads) gate_kernel(GateArgs a) {
  const unsigned lane = threadIdx.x % 32;
  const unsigned rows = a.n * kVHeads;
  const float4 nw = reinterpret_cast<const float4*>(a.norm_w)[lane];
  for (unsigned r = a.t0 * kVHeads + (blockIdx.x * kGateThreads + threadIdx.x) / 32; r < rows;
       r += gridDim.x * (kGateThreads / 32)) {
    const unsigned t = r / kVHeads, h = r % kVHeads;
    float4* o4 = reinterpret_cast<float4*>(a.out + size_t(r) * kDim) + lane;
    const float4 z = *(reinterpret_cast<const float4*>(a.z + size_t(t) * a.zab_stride +
                                                       h * kDim) + lane);
    float4 o = *o4;
    float ss = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float rr = rsqrtf(ss * (1.0f / kDim) + a.eps);
    o.x = o.x * rr * nw.x * silu(z.x);
    o.y = o.y * rr * nw.y * silu(z.y);
    o.z = o.z * rr * nw.z * silu(z.z);
    o.w = o.w * rr * nw.w * silu(z.w);
    *o4 = o;
  }
}

}  // namespace miso::fast::dnpf
