#pragma once

// Sparse MoE block for a chunk of n tokens, the drop-in for the reference's
// kernels/moe_prefill.hpp (interface :28-33, :74-91, :116-126, :223-235, :350-360, :496-500;
// launched by src/engine/moe.hip:95-127). Routing is the decode routing, token by token:
//   moe_router_batch: logits [n][257] through the decode router's row function (bitwise equal).
//   moe_topk_batch:   per token the decode top 8 (same function) plus slot 8 = the shared expert
//                     (id 256, weight sigmoid(logits[256])). Assignment a = 9 t + k.
//   moe_group:        a stable counting sort of the 9 n assignments by expert id (0..256), cut
//                     into tasks of at most kTaskTok assignments of one expert:
//                     {expert, first index into order, count, 0}.
//   moe_gate_up_grouped: per (task, half of the 512 rows): one thread per row pair (gate, up),
//                     the row's Q4_K weights expanded once per 256-block and applied to every
//                     assignment of the task; ah = FP16(SiLU(gate) * up), as = per-16 sums of ah.
//   moe_down_grouped: per (task, eighth of the 2048 rows): one thread per down row (K = 512),
//                     part[a][r] = weight[a] * down_e[r] . ah[a].
//   moe_combine:      out[t] = sum over the 9 slots of part[9 t + k], in slot order.

#include <cuda_fp16.h>

#include <cstddef>
#include <cstdint>

#include "f16_ptr.hpp"
#include "moe_decode.hpp"

namespace miso::kernels {

namespace moe {
inline constexpr int kTaskTok = 16;  // assignments per grouped task
}  // namespace moe

struct MoeRouterBatchParams {
  const std::uint16_t* w;  // [257][2048] BF16
  const float* x;          // [n_tok][2048]
  float* logits;           // [n_tok][257]
  unsigned n_tok;
};

// One block per token; its warps stride over the 257 rows.
__host__ __device__ inline unsigned moe_router_batch_items(unsigned n_tok, int block) {
  (void)block;
  return n_tok;
}

template <int kBlock>
__device__ inline void moe_router_batch_op(const MoeRouterBatchParams& p, unsigned first,
                                           unsigned count) {
  constexpr unsigned kWarps = kBlock / kWave;
  for (unsigned t = first + blockIdx.x; t < first + count; t += gridDim.x) {
    const float* x = p.x + std::size_t{t} * moe::kHidden;
    for (unsigned r = threadIdx.x / kWave; r <= moe::kExperts; r += kWarps) {
      const float v = moe_detail::router_row(p.w + std::size_t{r} * moe::kHidden, x);
      if (threadIdx.x % kWave == 0)
        p.logits[std::size_t{t} * (moe::kExperts + 1) + r] = v;
    }
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) moe_router_batch_kernel(MoeRouterBatchParams p) {
  moe_router_batch_op<kBlock>(p, 0, p.n_tok);
}

struct MoeTopkBatchParams {
  const float* logits;  // [n_tok][257]
  int* ids;             // [n_tok][9]
  float* weights;       // [n_tok][9]
  unsigned n_tok;
};

// Tokens [first, first + count), one block each (warp 0 works).
template <int kBlock>
__device__ inline void moe_topk_batch_op(const MoeTopkBatchParams& p, unsigned first,
                                         unsigned count) {
  for (unsigned t = first + blockIdx.x; t < first + count; t += gridDim.x) {
    if (threadIdx.x >= kWave)
      continue;
    const float* l = p.logits + std::size_t{t} * (moe::kExperts + 1);
    int id[moe::kTopK];
    float w[moe::kTopK];
    moe_detail::topk(l, id, w);
    const std::size_t a = std::size_t{t} * moe::kSlots;
    if (threadIdx.x < moe::kTopK)
      p.ids[a + threadIdx.x] = id[threadIdx.x], p.weights[a + threadIdx.x] = w[threadIdx.x];
    if (threadIdx.x == moe::kTopK) {
      p.ids[a + moe::kTopK] = static_cast<int>(moe::kExperts);
      p.weights[a + moe::kTopK] = moe_detail::sigmoid(l[moe::kExperts]);
    }
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) moe_topk_batch_kernel(MoeTopkBatchParams p) {
  moe_topk_batch_op<kBlock>(p, 0, p.n_tok);
}

struct MoeGroupParams {
  const int* ids;  // [n_tok][9]
  int* order;      // [9 n_tok]: assignments sorted by expert
  int4* tasks;     // {expert, first index into order, count, 0}
  int* n_tasks;
  unsigned n_tok;
};

// Upper bound of the task count: sum over the 257 ids of ceil(c_e / 16) <= 9 n / 16 + 257.
__host__ __device__ inline unsigned moe_max_tasks(unsigned n_tok) {
  return n_tok * moe::kSlots / moe::kTaskTok + moe::kExperts + 1;
}

// One block of kBlock >= 257 threads. Thread e owns expert e: it counts, then (tile by tile of
// kBlock assignments staged in shared memory) appends the assignments of expert e in index order,
// which makes the sort stable and deterministic. Ids outside 0..256 are dropped.
template <int kBlock>
__device__ inline void moe_group_op(const MoeGroupParams& p) {
  constexpr unsigned kIds = moe::kExperts + 1;
  static_assert(kBlock >= static_cast<int>(kIds), "one thread per expert id");
  __shared__ int tile[kBlock];
  __shared__ unsigned cnt[kIds], start[kIds], task0[kIds + 1];
  const unsigned e = threadIdx.x, n_asg = p.n_tok * moe::kSlots;
  if (e < kIds)
    cnt[e] = 0;
  __syncthreads();
  for (unsigned a = threadIdx.x; a < n_asg; a += kBlock) {
    const int id = p.ids[a];
    if (id >= 0 && id < static_cast<int>(kIds))
      atomicAdd(&cnt[id], 1u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned s = 0, t = 0;
    for (unsigned i = 0; i < kIds; ++i) {
      start[i] = s, task0[i] = t;
      s += cnt[i];
      t += (cnt[i] + moe::kTaskTok - 1) / moe::kTaskTok;
    }
    task0[kIds] = t;
    *p.n_tasks = static_cast<int>(t);
  }
  __syncthreads();
  unsigned cursor = e < kIds ? start[e] : 0;
  for (unsigned a0 = 0; a0 < n_asg; a0 += kBlock) {
    tile[threadIdx.x] = a0 + threadIdx.x < n_asg ? p.ids[a0 + threadIdx.x] : -1;
    __syncthreads();
    if (e < kIds) {
      const unsigned n = min(static_cast<unsigned>(kBlock), n_asg - a0);
      for (unsigned i = 0; i < n; ++i)
        if (tile[i] == static_cast<int>(e))
          p.order[cursor++] = static_cast<int>(a0 + i);
    }
    __syncthreads();
  }
  if (e < kIds) {
    for (unsigned q = 0; task0[e] + q < task0[e + 1]; ++q) {
      const unsigned first = start[e] + q * moe::kTaskTok;
      const unsigned c = min(static_cast<unsigned>(moe::kTaskTok), cnt[e] - q * moe::kTaskTok);
      p.tasks[task0[e] + q] = make_int4(static_cast<int>(e), static_cast<int>(first),
                                        static_cast<int>(c), 0);
    }
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) moe_group_kernel(MoeGroupParams p) {
  moe_group_op<kBlock>(p);
}

struct MoeGateUpGroupedParams {
  const std::uint8_t* gate_exps;  // Q4_K r1, [256][512 rows], K = 2048
  const std::uint8_t* up_exps;
  const std::uint8_t* gate_sh;  // Q4_K r1, [512 rows]
  const std::uint8_t* up_sh;
  F16In xh;          // [n_tok][2048]
  const float* xs;   // [n_tok][64]: per-32 sums of xh
  const int* order;
  const int4* tasks;
  const int* n_tasks;
  F16Out ah;  // [9 n_tok][512]: SiLU(gate) * up, rounded to FP16
  float* as;  // [9 n_tok][32]: per-16 sums of ah
};

namespace moe_detail {

// (d * sc, dmin * m) of sub-block j (0..7) of a Q4_K r1 block whose 16-byte header is h.
__device__ __forceinline__ float2 q4k_sub_scale(const uint4& h, unsigned j) {
  const unsigned bit = 24 * (j / 2);
  const uint32_t lo_w = gemv::word(h, 1 + bit / 32);
  const uint32_t hi_w = bit / 32 + 2 < 4 ? gemv::word(h, 2 + bit / 32) : 0u;
  const uint32_t f = __funnelshift_r(lo_w, hi_w, bit % 32) >> (12 * (j % 2));
  return make_float2(gemv::f16_bits(h.x & 0xFFFFu) * gemv::small_int_f(f & 63u),
                     gemv::f16_bits(h.x >> 16) * gemv::small_int_f((f >> 6) & 63u));
}

// sum over l < 32 of q[l] x[a][l] for the 32 elements of sub-block j of kM Q4_K r1 blocks (nibble
// bytes qs[m]: element l is byte 32 (j / 2) + l, low nibble for even j), for every assignment a
// (x rows of stride `ld` floats, 16-byte aligned). One pass over the activations serves all kM
// weight rows.
template <unsigned kT, int kM>
__device__ __forceinline__ void q4k_sub_dot(const std::uint8_t* const (&qs)[kM], unsigned j,
                                            const float* x, unsigned ld, float (&out)[kM][kT]) {
  uint4 q[kM][2];
#pragma unroll
  for (int m = 0; m < kM; ++m) {
    q[m][0] = __ldg(reinterpret_cast<const uint4*>(qs[m] + 32 * (j / 2)));
    q[m][1] = __ldg(reinterpret_cast<const uint4*>(qs[m] + 32 * (j / 2) + 16));
  }
  const unsigned sh = 4 * (j % 2);
#pragma unroll
  for (int m = 0; m < kM; ++m)
#pragma unroll
    for (unsigned a = 0; a < kT; ++a)
      out[m][a] = 0.0f;
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    float qn[kM][4];
#pragma unroll
    for (int m = 0; m < kM; ++m) {
      const uint32_t wd = gemv::word(q[m][v / 4], v % 4);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        qn[m][e] = gemv::small_int_f((wd >> (8 * e + sh)) & 15u);
    }
#pragma unroll
    for (unsigned a = 0; a < kT; ++a) {
      const float4 xv = *reinterpret_cast<const float4*>(x + a * ld + 4 * v);
#pragma unroll
      for (int m = 0; m < kM; ++m)
        out[m][a] += qn[m][0] * xv.x + qn[m][1] * xv.y + qn[m][2] * xv.z + qn[m][3] * xv.w;
    }
  }
}

}  // namespace moe_detail

// Work items [first, first + count) of 2 per task (256 row pairs each), up to 2 * n_tasks.
template <int kBlock>
__device__ inline void moe_gate_up_grouped_op(const MoeGateUpGroupedParams& p, unsigned first,
                                              unsigned count) {
  static_assert(kBlock == 256, "one thread per row of a half of the 512 rows");
  constexpr unsigned kT = moe::kTaskTok, K = moe::kHidden;
  constexpr std::size_t kRow = gemv::q4k_row_bytes(K);
  __shared__ __align__(16) float xs[kT][256];
  __shared__ float xsum[kT][8];
  for (unsigned item = first + blockIdx.x; item < first + count; item += gridDim.x) {
    const unsigned task = item / 2, half = item % 2;
    if (task >= static_cast<unsigned>(*p.n_tasks))
      return;  // uniform over the block; later items are larger
    const int4 tk = p.tasks[task];
    const unsigned e = static_cast<unsigned>(tk.x), n = static_cast<unsigned>(tk.z);
    const unsigned r = 256 * half + threadIdx.x;
    const std::size_t row = e < moe::kExperts ? std::size_t{e} * moe::kFf + r : r;
    const std::uint8_t* gw = (e < moe::kExperts ? p.gate_exps : p.gate_sh) + row * kRow;
    const std::uint8_t* uw = (e < moe::kExperts ? p.up_exps : p.up_sh) + row * kRow;
    float ga[kT] = {}, ua[kT] = {};
    for (unsigned kb = 0; kb < K / 256; ++kb) {
      __syncthreads();  // previous block's activations are consumed
      for (unsigned i = threadIdx.x; i < kT * 256 / 8; i += kBlock) {
        const unsigned a = i / 32, c = i % 32;  // assignment a, 8-element chunk c
        float4 lo = make_float4(0, 0, 0, 0), hi = lo;
        if (a < n) {
          const unsigned t = static_cast<unsigned>(p.order[tk.y + a]) / moe::kSlots;
          const uint4 v = *reinterpret_cast<const uint4*>(p.xh.p + std::size_t{t} * K + 256 * kb + 8 * c);
          const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
          const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
          const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
          const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
          lo = make_float4(f0.x, f0.y, f1.x, f1.y), hi = make_float4(f2.x, f2.y, f3.x, f3.y);
          if (c % 4 == 0)
            xsum[a][c / 4] = p.xs[std::size_t{t} * (K / 32) + 8 * kb + c / 4];
        } else if (c % 4 == 0) {
          xsum[a][c / 4] = 0.0f;
        }
        *reinterpret_cast<float4*>(&xs[a][8 * c]) = lo;
        *reinterpret_cast<float4*>(&xs[a][8 * c + 4]) = hi;
      }
      __syncthreads();
      const std::uint8_t* gblk = gw + std::size_t{kb} * 144;
      const std::uint8_t* ublk = uw + std::size_t{kb} * 144;
      const uint4 gh = __ldg(reinterpret_cast<const uint4*>(gblk));
      const uint4 uh = __ldg(reinterpret_cast<const uint4*>(ublk));
      const std::uint8_t* const qs[2] = {gblk + 16, ublk + 16};
      for (unsigned j = 0; j < 8; ++j) {
        float q[2][kT];
        const float2 gs = moe_detail::q4k_sub_scale(gh, j), us = moe_detail::q4k_sub_scale(uh, j);
        moe_detail::q4k_sub_dot<kT, 2>(qs, j, &xs[0][32 * j], 256, q);
#pragma unroll
        for (unsigned a = 0; a < kT; ++a) {
          ga[a] += gs.x * q[0][a] - gs.y * xsum[a][j];
          ua[a] += us.x * q[1][a] - us.y * xsum[a][j];
        }
      }
    }
#pragma unroll
    for (unsigned a = 0; a < kT; ++a) {
      const float h = gemv::round_f16(moe_detail::silu(ga[a]) * ua[a]);
      float s = h;  // per-16 sums over 16 consecutive rows = 16 consecutive lanes
#pragma unroll
      for (int off = 8; off > 0; off >>= 1)
        s += __shfl_xor_sync(0xffffffffu, s, off);
      if (a < n) {
        const std::size_t asg = static_cast<unsigned>(p.order[tk.y + a]);
        p.ah.p[asg * moe::kFf + r] = __float2half_rn(h);
        if (threadIdx.x % 16 == 0)
          p.as[asg * (moe::kFf / 16) + r / 16] = s;
      }
    }
  }
}

template <int kBlock>
__global__ void __launch_bounds__(kBlock) moe_gate_up_grouped_kernel(MoeGateUpGroupedParams p) {
  moe_gate_up_grouped_op<kBlock>(p, 0, 2 * static_cast<unsigned>(*p.n_tasks));
}

struct MoeDownGroupedParams {
  const std::uint8_t* down_exps;  // r1, [256][2048 rows], K = 512
  const std::uint8_t* down_sh;    // r1, [2048 rows]
  F16In ah;                       // [9 n_tok][512]
  const float* as;                // [9 n_tok][32]
  const float* weights;           // [9 n_tok]
  const int* order;
  const int4* tasks;
  const int* n_tasks;
  float* part;  // [9 n_tok][2048]: weight * down(ah)
};

// Work items [first, first + count) of 8 per task (256 output rows each), up to 8 * n_tasks.
template <QType T, int kBlock>
__device__ inline void moe_down_grouped_op(const MoeDownGroupedParams& p, unsigned first,
                                           unsigned count) {
  static_assert(kBlock == 256, "one thread per output row of an eighth of the 2048");
  constexpr unsigned kT = moe::kTaskTok, K = moe::kFf;
  constexpr std::size_t kRow = T == QType::Q4K ? gemv::q4k_row_bytes(K) : gemv::q6k_row_bytes(K);
  __shared__ __align__(16) float hs[kT][K];
  __shared__ float hsum[kT][K / 16];
  for (unsigned item = first + blockIdx.x; item < first + count; item += gridDim.x) {
    const unsigned task = item / 8, part = item % 8;
    if (task >= static_cast<unsigned>(*p.n_tasks))
      return;
    const int4 tk = p.tasks[task];
    const unsigned e = static_cast<unsigned>(tk.x), n = static_cast<unsigned>(tk.z);
    const unsigned r = 256 * part + threadIdx.x;
    __syncthreads();  // the previous item's activations are consumed
    for (unsigned i = threadIdx.x; i < kT * K / 8; i += kBlock) {
      const unsigned a = i / (K / 8), c = i % (K / 8);
      float4 lo = make_float4(0, 0, 0, 0), hi = lo;
      if (a < n) {
        const std::size_t asg = static_cast<unsigned>(p.order[tk.y + a]);
        const uint4 v = *reinterpret_cast<const uint4*>(p.ah.p + asg * K + 8 * c);
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
        const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
        const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
        lo = make_float4(f0.x, f0.y, f1.x, f1.y), hi = make_float4(f2.x, f2.y, f3.x, f3.y);
        if (c % 2 == 0)
          hsum[a][c / 2] = p.as[asg * (K / 16) + c / 2];
      } else if (c % 2 == 0) {
        hsum[a][c / 2] = 0.0f;
      }
      *reinterpret_cast<float4*>(&hs[a][8 * c]) = lo;
      *reinterpret_cast<float4*>(&hs[a][8 * c + 4]) = hi;
    }
    __syncthreads();
    const std::size_t row = e < moe::kExperts ? std::size_t{e} * moe::kHidden + r : r;
    const std::uint8_t* w = (e < moe::kExperts ? p.down_exps : p.down_sh) + row * kRow;
    float acc[kT] = {};
    if (T == QType::Q4K) {
      for (unsigned b = 0; b < K / 256; ++b) {
        const std::uint8_t* blk = w + std::size_t{b} * 144;
        const uint4 h = __ldg(reinterpret_cast<const uint4*>(blk));
        const std::uint8_t* const qs[1] = {blk + 16};
        for (unsigned j = 0; j < 8; ++j) {
          float q[1][kT];
          moe_detail::q4k_sub_dot<kT, 1>(qs, j, &hs[0][256 * b + 32 * j], K, q);
          const float2 sm = moe_detail::q4k_sub_scale(h, j);
          const unsigned g16 = (256 * b + 32 * j) / 16;
#pragma unroll
          for (unsigned a = 0; a < kT; ++a)
            acc[a] += sm.x * q[0][a] - sm.y * (hsum[a][g16] + hsum[a][g16 + 1]);
        }
      }
    } else {
      // Q6_K r1 row of 2 blocks: ql at 128 b, qh at 256 + 64 b, scales at 384 + 16 b, d at 416 + 2b.
      constexpr unsigned nb = K / 256;
      for (unsigned b = 0; b < nb; ++b) {
        const float d = gemv::f16_bits(*reinterpret_cast<const uint16_t*>(w + nb * 208 + 2 * b));
        const int8_t* sc = reinterpret_cast<const int8_t*>(w + nb * 192 + 16 * b);
        for (unsigned g = 0; g < 16; ++g) {  // 16-element groups: half n, quarter u, l0 = 16 (g % 2)
          const unsigned n = g / 8, u = (g % 8) / 2, l0 = 16 * (g % 2);
          const uint4 ql = __ldg(reinterpret_cast<const uint4*>(w + 128 * b + 64 * n + 32 * (u % 2) + l0));
          const uint4 qh = __ldg(reinterpret_cast<const uint4*>(w + nb * 128 + 64 * b + 32 * n + l0));
          const float ds = d * static_cast<float>(sc[8 * n + g % 2 + 2 * u]);
          const unsigned e0 = 256 * b + 128 * n + 32 * u + l0;  // first element of the group
          float q[kT] = {};
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const uint32_t a4 = gemv::word(ql, v), h4 = gemv::word(qh, v);
            float qn[4];
#pragma unroll
            for (int m = 0; m < 4; ++m)
              qn[m] = gemv::q6_f(((a4 >> (8 * m + 4 * (u / 2))) & 15u) |
                                 ((h4 >> (8 * m + 2 * u)) & 3u) << 4);
#pragma unroll
            for (unsigned a = 0; a < kT; ++a) {
              const float4 x = *reinterpret_cast<const float4*>(&hs[a][e0 + 4 * v]);
              q[a] += qn[0] * x.x + qn[1] * x.y + qn[2] * x.z + qn[3] * x.w;
            }
          }
#pragma unroll
          for (unsigned a = 0; a < kT; ++a)
            acc[a] += ds * q[a];
        }
      }
    }
#pragma unroll
    for (unsigned a = 0; a < kT; ++a) {
      if (a < n) {
        const std::size_t asg = static_cast<unsigned>(p.order[tk.y + a]);
        p.part[asg * moe::kHidden + r] = p.weights[asg] * acc[a];
      }
    }
  }
}

template <QType T, int kBlock>
__global__ void __launch_bounds__(kBlock) moe_down_grouped_kernel(MoeDownGroupedParams p) {
  moe_down_grouped_op<T, kBlock>(p, 0, 8 * static_cast<unsigned>(*p.n_tasks));
}

struct MoeCombineParams {
  const float* part;  // [9 n_tok][2048], weighted slot outputs
  float* out;         // [n_tok][2048]
  unsigned n_tok;
};

// Float4 elements [first, first + count) of n_tok * 512.
__device__ inline void moe_combine_op(const MoeCombineParams& p, unsigned first, unsigned count) {
  constexpr unsigned kVec = moe::kHidden / 4;
  for (unsigned i = first + blockIdx.x * blockDim.x + threadIdx.x; i < first + count;
       i += gridDim.x * blockDim.x) {
    const unsigned t = i / kVec, c = i % kVec;
    const float4* src = reinterpret_cast<const float4*>(p.part) + std::size_t{t} * moe::kSlots * kVec + c;
    float4 s = src[0];
#pragma unroll
    for (unsigned k = 1; k < moe::kSlots; ++k) {
      const float4 v = src[k * kVec];
      s.x += v.x, s.y += v.y, s.z += v.z, s.w += v.w;
    }
    reinterpret_cast<float4*>(p.out)[i] = s;
  }
}

__global__ void __launch_bounds__(256) moe_combine_kernel(MoeCombineParams p) {
  moe_combine_op(p, 0, p.n_tok * (moe::kHidden / 4));
}

}  // namespace miso::kernels
