#pragma once

// Batched split-K GQA decode for B200 (sm_100a): the fast path behind miso_attn_decode().
//
// Work: for every (sequence b, KV head h) segment, core = softmax(q K^T / 16) V * sigmoid(gate)
// for the 8 query heads that share KV head h. Decode reads each K/V row exactly once and does
// 8 FLOP per KV byte, so the kernel is HBM-bound; its job is to keep enough bytes in flight and
// spend as few issue slots as possible per byte.
//
// Decomposition (stream-K): the key axis of all segments is cut into 64-key tiles, listed segment
// by segment; CTA c of P (one per SM) takes the contiguous tile range [c T / P, (c + 1) T / P),
// so every SM streams the same number of bytes whatever the length mix. A segment that lies in
// one CTA is finished there; a segment cut across CTAs is finished by the last of its CTAs to
// arrive (per-segment counter in scratch), which merges the partial (max, sum, output) triples in
// CTA order — no spin-waits, deterministic results.
//
// Per CTA: warp 8 is the producer (one lane issues TMA loads of four 64x64 fp16 boxes of K and
// four of V per tile into a 3-stage ring, 128-byte swizzled); warps 0-7 consume. Tile i goes to
// warp group i & 1, and warp w of the group takes keys [16 (w % 4), +16) of it. Each consumer warp
// runs its own online softmax over its keys (tensor cores, m16n8k16, f16 in / f32 accumulate):
//   S^T[16 keys][8 heads] = K[16][256] . Q^T           (Q split into fp16 hi + lo: two MMAs)
//   O^T[256][8 heads]    += V^T[256][16 keys] . P^T    (P split into fp16 hi + lo: two MMAs)
// K is exactly fp16 (the cache), so hi/lo splitting keeps the fp32 reference accuracy
// (relative L2 ~1e-6 vs fp64). The eight warps' states are merged through shared memory at the
// end of each segment.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../common/device.cuh"

namespace miso::fast::decode {

constexpr int kQHeads = 16, kKvHeads = 2, kDim = 256, kGroup = 8;
constexpr int kTile = 64;                      // keys per pipeline stage
constexpr int kStages = 3;
constexpr int kBars = 6;  // lcm(kStages, 2)
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;      // + producer warp
constexpr int kBoxBytes = 64 * 128;            // TMA box: 64 rows x 64 dims fp16
constexpr int kHalfStage = 4 * kBoxBytes;      // K (or V) of one tile
constexpr int kStageBytes = 2 * kHalfStage;    // 64 KiB
constexpr int kMaxBatch = 1024;
constexpr unsigned kMinTiles = 4;              // fewest tiles a working CTA takes
constexpr unsigned kMaxCtas = 256;             // grid limit: the merge weights fit one slot
constexpr int kSlotRow = 260;                  // padded [head][dim] row of a merge slot (floats)
constexpr int kSlotFloats = kGroup * kSlotRow + kGroup;  // o[8][260] then l[8]
constexpr int kPartFloats = 2 * kGroup + kGroup * kDim;  // m[8], l[8], o[8][256]
static_assert(kMaxCtas * kGroup + kGroup <= kSlotFloats, "merge weights [P][8] + L[8] in a slot");
static_assert(kMaxCtas <= kSlotFloats, "merge offsets [P] in the other slot");

struct Args {
  const float* q;
  const float* qg;
  const int64_t* kv_row;
  const int32_t* lens;
  float* core;
  int* counters;  // [2 * batch]
  float* parts;   // [2 * gridDim.x][kPartFloats]
  unsigned batch;
  unsigned qg_stride;
};

struct Smem {
  // stages first: must be 1024-byte aligned for the 128B swizzle
  uint4 qfrag[16][32];  // per k-step and lane: Q^T B fragments {hi.b01, hi.b23, lo.b01, lo.b23}
  float slot[2][kSlotFloats];
  float red_m[kConsumerWarps][kGroup];
  int seq_start[kMaxBatch + 1];
  // Barriers are indexed by tile % kBars (kBars = lcm(kStages, 2 warp groups)): every barrier is
  // then used by one warp group only, in tile order, so a parity wait never has to tell a phase
  // from the one two steps before it.
  uint64_t full[kBars], empty[kBars];
  int abort_flag;
  int is_last;
};

constexpr size_t kSmemBytes = 1024 + size_t(kStages) * kStageBytes + sizeof(Smem);

__device__ __forceinline__ unsigned owner_of(unsigned tile, unsigned T, unsigned P) {
  return static_cast<unsigned>((static_cast<uint64_t>(tile + 1) * P - 1) / T);
}

__device__ __forceinline__ unsigned range_begin(unsigned c, unsigned T, unsigned P) {
  return static_cast<unsigned>(static_cast<uint64_t>(c) * T / P);
}

// Largest b with seq_start[b] <= tile (seq_start is non-decreasing, seq_start[0] = 0).
__device__ __forceinline__ unsigned seq_of(const int* seq_start, unsigned batch, unsigned tile) {
  unsigned lo = 0, hi = batch;  // answer in [lo, hi)
  while (hi - lo > 1) {
    const unsigned mid = (lo + hi) / 2;
    if (static_cast<unsigned>(seq_start[mid]) <= tile)
      lo = mid;
    else
      hi = mid;
  }
  return lo;
}

__device__ __forceinline__ float fast_exp(float x) { return __expf(x); }

__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = base;
  Smem& sm = *reinterpret_cast<Smem*>(base + size_t(kStages) * kStageBytes);
  const unsigned tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const unsigned c = blockIdx.x;
  const float kNegInf = -__int_as_float(0x7f800000);

  // ---- tile prefix over sequences: seq_start[b] = sum_{b' < b} 2 ceil(len / 64) ----------------
  if (warp == 0) {
    const unsigned per = (a.batch + 31) / 32;
    const unsigned b0 = lane * per, b1 = min(a.batch, b0 + per);
    int local = 0;
    for (unsigned b = b0; b < b1; ++b) {
      const int len = max(a.lens[b], 0);
      local += 2 * ((len + kTile - 1) / kTile);
    }
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= static_cast<unsigned>(off))
        incl += y;
    }
    int run = incl - local;
    for (unsigned b = b0; b < b1; ++b) {
      sm.seq_start[b] = run;
      const int len = max(a.lens[b], 0);
      run += 2 * ((len + kTile - 1) / kTile);
    }
    if (lane == 31)
      sm.seq_start[a.batch] = incl;
  }
  if (tid == 0) {
    for (int s = 0; s < kBars; ++s) {
      dev::mbar_init(dev::smem_u32(&sm.full[s]), 1);
      dev::mbar_init(dev::smem_u32(&sm.empty[s]), 4);
    }
    sm.abort_flag = 0;
    dev::mbar_init_fence();
  }
  __syncthreads();

  const unsigned T = static_cast<unsigned>(sm.seq_start[a.batch]);
  // At least kMinTiles tiles per working CTA: with fewer, half of the consumer warps idle and a
  // segment is cut into more partials than its bytes justify (small batches, short contexts).
  // CTAs c >= P get an empty range.
  const unsigned P = max(1u, min(gridDim.x, T / kMinTiles));
  const unsigned t_begin = (T == 0 || c >= P) ? T : range_begin(c, T, P);
  const unsigned t_end = (T == 0 || c >= P) ? T : range_begin(c + 1, T, P);

  // ---------------------------------------------------------------------------------- producer
  if (warp == kConsumerWarps) {
    if (lane == 0 && t_begin < t_end) {
      unsigned issued = 0;  // tiles whose loads have been issued
      dev::tma_prefetch_desc(&kmap);
      dev::tma_prefetch_desc(&vmap);
      const uint64_t policy = dev::policy_evict_first();
      unsigned b = seq_of(sm.seq_start, a.batch, t_begin);
      for (unsigned i = t_begin; i < t_end; ++i) {
        while (static_cast<unsigned>(sm.seq_start[b + 1]) <= i)
          ++b;
        const unsigned nt = (sm.seq_start[b + 1] - sm.seq_start[b]) / 2;
        const unsigned local = i - sm.seq_start[b], kvh = local / nt, j = local - kvh * nt;
        const int y = static_cast<int>(a.kv_row[2 * b + kvh] + int64_t(j) * kTile);
        const unsigned k = i - t_begin, s = k % kStages;
        const uint32_t full = dev::smem_u32(&sm.full[k % kBars]);
        // Stage s is free once tile k - kStages has been consumed (its group's empty barrier).
        if (k >= kStages &&
            !dev::mbar_wait(dev::smem_u32(&sm.empty[(k - kStages) % kBars]),
                            ((k - kStages) / kBars) & 1, 0x11)) {
          sm.abort_flag = 1;
          break;
        }
        if (*reinterpret_cast<volatile int*>(&sm.abort_flag))
          break;
        issued = k + 1;
        dev::mbar_arrive_expect_tx(full, kStageBytes);
        const uint32_t kdst = dev::smem_u32(stages + size_t(s) * kStageBytes);
        const uint32_t vdst = kdst + kHalfStage;
#pragma unroll
        for (int box = 0; box < 4; ++box) {
          dev::tma_load_2d_hint(kdst + box * kBoxBytes, &kmap, box * 64, y, full, policy);
          dev::tma_load_2d_hint(vdst + box * kBoxBytes, &vmap, box * 64, y, full, policy);
        }
      }
      if (*reinterpret_cast<volatile int*>(&sm.abort_flag)) {
        // Let the copies of the last (up to kStages) issued tiles land before the CTA can exit.
        for (unsigned k = issued > kStages ? issued - kStages : 0; k < issued; ++k)
          dev::mbar_wait(dev::smem_u32(&sm.full[k % kBars]), (k / kBars) & 1, 0x13);
      }
    }
    __syncwarp();  // the producer lane rejoins its warp before the block-wide barrier
  } else {

  // ---------------------------------------------------------------------------------- consumers
  // Sequences with no keys produce zeros; CTA min(owner, P - 1) of their (empty) tile index
  // writes them.
  for (unsigned b = 0; b < a.batch; ++b) {
    if (sm.seq_start[b + 1] != sm.seq_start[b])
      continue;
    const unsigned at = sm.seq_start[b];
    const unsigned own = (T == 0 || at >= T) ? (T == 0 ? 0 : P - 1) : owner_of(at, T, P);
    if (own != c)
      continue;
    for (unsigned i = tid; i < kQHeads * kDim; i += kConsumers)
      a.core[size_t(b) * kQHeads * kDim + i] = 0.0f;
  }
  if (t_begin < t_end) {

  const unsigned group = warp / 4, slab = (warp % 4) * 16;
  const unsigned g = lane / 4, tq = lane % 4;  // fragment row group / thread-in-group
  const unsigned mi = lane / 8, ri = lane % 8;  // ldmatrix: matrix index / row within matrix

  float o[16][4];
  float m0 = kNegInf, m1 = kNegInf, l0 = 0.0f, l1 = 0.0f;

  unsigned cur_b = ~0u, cur_kvh = 0;
  unsigned b = seq_of(sm.seq_start, a.batch, t_begin);

  // Merges the eight warps' states of segment (sb, skvh) and writes the output or the partial.
  auto finish = [&](unsigned sb, unsigned skvh) {
    // Sum l over the 8 row groups of the warp.
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (g == 0)
      sm.red_m[warp][2 * tq] = m0, sm.red_m[warp][2 * tq + 1] = m1;
    dev::named_bar_sync(1, kConsumers);
    float M0 = kNegInf, M1 = kNegInf;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      M0 = fmaxf(M0, sm.red_m[w][2 * tq]);
      M1 = fmaxf(M1, sm.red_m[w][2 * tq + 1]);
    }
    const float sc0 = m0 == kNegInf ? 0.0f : fast_exp(m0 - M0);
    const float sc1 = m1 == kNegInf ? 0.0f : fast_exp(m1 - M1);
    l0 *= sc0, l1 *= sc1;
#pragma unroll
    for (int mb = 0; mb < 16; ++mb)
      o[mb][0] *= sc0, o[mb][1] *= sc1, o[mb][2] *= sc0, o[mb][3] *= sc1;

    auto put = [&](int slot) {
      float* sl = sm.slot[slot];
#pragma unroll
      for (int mb = 0; mb < 16; ++mb) {
        const int d = mb * 16 + g;
        sl[(2 * tq) * kSlotRow + d] = o[mb][0];
        sl[(2 * tq + 1) * kSlotRow + d] = o[mb][1];
        sl[(2 * tq) * kSlotRow + d + 8] = o[mb][2];
        sl[(2 * tq + 1) * kSlotRow + d + 8] = o[mb][3];
      }
      if (g == 0)
        sl[kGroup * kSlotRow + 2 * tq] = l0, sl[kGroup * kSlotRow + 2 * tq + 1] = l1;
    };
    auto take = [&](int slot) {
      const float* sl = sm.slot[slot];
#pragma unroll
      for (int mb = 0; mb < 16; ++mb) {
        const int d = mb * 16 + g;
        o[mb][0] += sl[(2 * tq) * kSlotRow + d];
        o[mb][1] += sl[(2 * tq + 1) * kSlotRow + d];
        o[mb][2] += sl[(2 * tq) * kSlotRow + d + 8];
        o[mb][3] += sl[(2 * tq + 1) * kSlotRow + d + 8];
      }
      l0 += sl[kGroup * kSlotRow + 2 * tq];
      l1 += sl[kGroup * kSlotRow + 2 * tq + 1];
    };
    // Tree: (w0+w4) (w1+w5), (w2+w6) (w3+w7), (w0+w2) (w1+w3), then slots hold w0 and w1.
    if (warp == 4 || warp == 5) put(warp - 4);
    dev::named_bar_sync(1, kConsumers);
    if (warp == 0 || warp == 1) take(warp);
    dev::named_bar_sync(1, kConsumers);
    if (warp == 6 || warp == 7) put(warp - 6);
    dev::named_bar_sync(1, kConsumers);
    if (warp == 2 || warp == 3) take(warp - 2);
    dev::named_bar_sync(1, kConsumers);
    if (warp == 2 || warp == 3) put(warp - 2);
    dev::named_bar_sync(1, kConsumers);
    if (warp == 0 || warp == 1) take(warp);
    dev::named_bar_sync(1, kConsumers);
    if (warp == 0 || warp == 1) put(warp);
    dev::named_bar_sync(1, kConsumers);

    // All 256 threads: combine slot 0 + slot 1, then finish or publish a partial.
    const unsigned seg = 2 * sb + skvh;
    const unsigned nt = (sm.seq_start[sb + 1] - sm.seq_start[sb]) / 2;
    const unsigned seg_first = sm.seq_start[sb] + skvh * nt, seg_last = seg_first + nt - 1;
    const unsigned c_first = owner_of(seg_first, T, P), c_last = owner_of(seg_last, T, P);
    const float* gate = a.qg + size_t(sb) * a.qg_stride + (skvh * kGroup) * 2 * kDim + kDim;
    float* out = a.core + (size_t(sb) * kQHeads + skvh * kGroup) * kDim;
    if (c_first == c_last) {
      for (unsigned i = tid; i < kGroup * kDim; i += kConsumers) {
        const unsigned h = i / kDim, d = i % kDim;
        const float ov = sm.slot[0][h * kSlotRow + d] + sm.slot[1][h * kSlotRow + d];
        const float L = sm.slot[0][kGroup * kSlotRow + h] + sm.slot[1][kGroup * kSlotRow + h];
        out[h * kDim + d] = ov / L / (1.0f + fast_exp(-gate[h * 2 * kDim + d]));
      }
    } else {
      const bool first_of_cta = seg_first <= t_begin;  // this segment holds tile t_begin
      float* part = a.parts + (size_t(2) * c + (first_of_cta ? 0 : 1)) * kPartFloats;
      for (unsigned i = tid; i < kGroup * kDim; i += kConsumers) {
        const unsigned h = i / kDim, d = i % kDim;
        part[2 * kGroup + i] = sm.slot[0][h * kSlotRow + d] + sm.slot[1][h * kSlotRow + d];
      }
      // The merged max of head h is the max over warps of red_m[w][h].
      if (tid < kGroup) {
        float M = kNegInf;
        for (int w = 0; w < kConsumerWarps; ++w)
          M = fmaxf(M, sm.red_m[w][tid]);
        part[tid] = M;
        part[kGroup + tid] = sm.slot[0][kGroup * kSlotRow + tid] + sm.slot[1][kGroup * kSlotRow + tid];
      }
      __threadfence();
      dev::named_bar_sync(1, kConsumers);
      if (warp == 0) {
        // CTAs between the segment's first and last owner may have empty ranges (T < P): warp 0
        // counts the non-empty ones (the range bounds take 64-bit divisions), lane 0 arrives.
        int parts = 0;
        for (unsigned cc = c_first + lane; cc <= c_last; cc += 32)
          parts += range_begin(cc, T, P) < range_begin(cc + 1, T, P);
        parts = __reduce_add_sync(0xffffffffu, parts);
        if (lane == 0) {
          const int prev = atomicAdd(&a.counters[seg], 1);
          sm.is_last = prev == parts - 1;
        }
      }
      dev::named_bar_sync(1, kConsumers);
      if (sm.is_last) {
        __threadfence();
        const unsigned seg_at_cfirst_start =
            static_cast<unsigned>(range_begin(c_first, T, P)) >= seg_first;
        // The segment's partials, in CTA order: CTA c_first + k wrote slot sl(k) (its second
        // slot when the segment is not the first of its range), or nothing for an empty range.
        const unsigned np = c_last - c_first + 1;
        // Partial k's slot index (or -1 for an empty range), computed once: the range bounds
        // take 64-bit divisions. The slots are free: this CTA's own result is in its partial.
        int* poff = reinterpret_cast<int*>(sm.slot[1]);  // [np]
        for (unsigned k = tid; k < np; k += kConsumers) {
          const unsigned cc = c_first + k;
          const unsigned sl = (cc > c_first || seg_at_cfirst_start) ? 0 : 1;
          poff[k] = range_begin(cc, T, P) == range_begin(cc + 1, T, P) ? -1 : int(2 * cc + sl);
        }
        dev::named_bar_sync(1, kConsumers);
        auto part_of = [&](unsigned k) -> const float* {
          const int o = poff[k];
          return o < 0 ? nullptr : a.parts + size_t(o) * kPartFloats;
        };
        // Weights: warp h finds head h's max over the partials, then w[k][h] = e^(m_k - M) and,
        // in lane 0, in partial order, L[h] = sum_k w[k][h] l_k.
        float* wts = sm.slot[0];             // [np][kGroup]
        float* Ls = sm.slot[0] + np * kGroup;  // [kGroup]
        // The partials' l values [np][kGroup], loaded by all lanes at once into the Q fragment
        // area (idle until the next segment), so that lane 0's ordered sum reads shared memory.
        float* lks = reinterpret_cast<float*>(sm.qfrag);
        {
          const unsigned h = warp;
          float M = kNegInf;
          for (unsigned k = lane; k < np; k += 32)
            if (const float* pp = part_of(k))
              M = fmaxf(M, __ldcg(pp + h));
#pragma unroll
          for (int off = 16; off > 0; off >>= 1)
            M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
          for (unsigned k = lane; k < np; k += 32) {
            const float* pp = part_of(k);
            const float mc = pp ? __ldcg(pp + h) : kNegInf;
            wts[k * kGroup + h] = mc == kNegInf ? 0.0f : fast_exp(mc - M);
            lks[k * kGroup + h] = pp ? __ldcg(pp + kGroup + h) : 0.0f;
          }
          __syncwarp();
          if (lane == 0) {
            float L = 0.0f;
            for (unsigned k = 0; k < np; ++k)
              if (poff[k] >= 0)
                L += wts[k * kGroup + h] * lks[k * kGroup + h];
            Ls[h] = L;
          }
        }
        dev::named_bar_sync(1, kConsumers);
        // Outputs: thread tid takes dimension tid of every head (eight independent sums, each
        // in partial order), so 8 x 4 loads are in flight at once.
        // Warp h takes head h, lane l dimensions [8 l, 8 l + 8): two 16-byte loads per partial.
        // Eight partials' values are loaded before any is accumulated; each output's sum still
        // runs over the partials in order.
        {
          const unsigned h = warp, d0 = 8 * lane;
          float ov[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            ov[e] = 0.0f;
          constexpr unsigned kBatch = 8;
#pragma unroll 1
          for (unsigned k0 = 0; k0 < np; k0 += kBatch) {
            float4 x[kBatch][2];
#pragma unroll
            for (unsigned j = 0; j < kBatch; ++j) {
              const float* pp = k0 + j < np ? part_of(k0 + j) : nullptr;
              const float4* src = reinterpret_cast<const float4*>(pp + 2 * kGroup + h * kDim + d0);
              x[j][0] = pp ? __ldcg(src) : make_float4(0.f, 0.f, 0.f, 0.f);
              x[j][1] = pp ? __ldcg(src + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (unsigned j = 0; j < kBatch; ++j)
              if (k0 + j < np && poff[k0 + j] >= 0) {
                const float w = wts[(k0 + j) * kGroup + h];
                ov[0] += w * x[j][0].x, ov[1] += w * x[j][0].y;
                ov[2] += w * x[j][0].z, ov[3] += w * x[j][0].w;
                ov[4] += w * x[j][1].x, ov[5] += w * x[j][1].y;
                ov[6] += w * x[j][1].z, ov[7] += w * x[j][1].w;
              }
          }
#pragma unroll
          for (int e = 0; e < 8; ++e)
            out[h * kDim + d0 + e] =
                ov[e] / Ls[h] / (1.0f + fast_exp(-gate[h * 2 * kDim + d0 + e]));
        }
        if (tid == 0)
          a.counters[seg] = 0;  // ready for the next call
      }
    }
    dev::named_bar_sync(1, kConsumers);  // slots / red_m / is_last free for the next segment
  };

  for (unsigned i = t_begin; i < t_end; ++i) {
    while (static_cast<unsigned>(sm.seq_start[b + 1]) <= i)
      ++b;
    const unsigned nt = (sm.seq_start[b + 1] - sm.seq_start[b]) / 2;
    const unsigned local = i - sm.seq_start[b], kvh = local / nt, j = local - kvh * nt;
    if (b != cur_b || kvh != cur_kvh) {
      if (cur_b != ~0u)
        finish(cur_b, cur_kvh);
      cur_b = b, cur_kvh = kvh;
      // This segment's 8 query heads as fp16 hi/lo B fragments (pre-scaled by 1/16, which is
      // exact), stored in fragment order so each lane later reads one 16-byte word per k-step.
      for (unsigned e = tid; e < 16 * 32; e += kConsumers) {
        const unsigned ks = e / 32, ln = e % 32, fg = ln / 4, ft = ln % 4;
        const float* qrow = a.q + (size_t(b) * kQHeads + kvh * kGroup + fg) * kDim + ks * 16;
        const float2 x01 = *reinterpret_cast<const float2*>(qrow + 2 * ft);
        const float2 x89 = *reinterpret_cast<const float2*>(qrow + 2 * ft + 8);
        uint4 f;
        dev::split_half2(x01.x * 0.0625f, x01.y * 0.0625f, f.x, f.z);
        dev::split_half2(x89.x * 0.0625f, x89.y * 0.0625f, f.y, f.w);
        sm.qfrag[ks][ln] = f;
      }
      dev::named_bar_sync(1, kConsumers);
#pragma unroll
      for (int mb = 0; mb < 16; ++mb)
        o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.0f;
      m0 = m1 = kNegInf, l0 = l1 = 0.0f;
    }
    const unsigned k = i - t_begin;
    if ((k & 1) != group)
      continue;
    const unsigned s = k % kStages;
    const uint32_t full = dev::smem_u32(&sm.full[k % kBars]);
    bool ok = !*reinterpret_cast<volatile int*>(&sm.abort_flag);
    if (ok && !dev::mbar_wait(full, (k / kBars) & 1, 0x12)) {
      sm.abort_flag = 1;
      ok = false;
    }
    uint8_t* kst = stages + size_t(s) * kStageBytes;
    uint8_t* vst = kst + kHalfStage;
    const int len = a.lens[b];
    const int key0 = int(j) * kTile + int(slab);  // first key of this warp's slab
    const int nvalid = min(16, len - key0);       // keys of the slab inside [0, len)
    if (ok && nvalid > 0) {
      if (nvalid < 16) {
        // Rows past len may hold anything (including NaN bit patterns): zero this slab's V rows
        // so that p = 0 times them stays 0.
        for (int r = nvalid; r < 16; ++r) {
          const unsigned row = slab + r;
          for (unsigned e = lane; e < 4 * 8; e += 32) {
            const unsigned box = e / 8, ch = e % 8;
            *reinterpret_cast<uint4*>(vst + box * kBoxBytes + dev::swz128(row, ch)) =
                make_uint4(0, 0, 0, 0);
          }
        }
        dev::fence_proxy_async_smem();
        __syncwarp();
      }
      // ---- S^T = K Q^T over 256 dims: four independent accumulator chains -----------------
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
      float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t kbase = dev::smem_u32(kst);
      const unsigned krow = slab + (mi & 1) * 8 + ri;
#pragma unroll 2
      for (int ks = 0; ks < 16; ks += 2) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        dev::ldsm_x4(kbase + (ks >> 2) * kBoxBytes + dev::swz128(krow, (ks & 3) * 2 + (mi >> 1)),
                     a0, a1, a2, a3);
        dev::ldsm_x4(kbase + ((ks + 1) >> 2) * kBoxBytes +
                         dev::swz128(krow, ((ks + 1) & 3) * 2 + (mi >> 1)),
                     b0, b1, b2, b3);
        const uint4 qa = sm.qfrag[ks][lane], qb = sm.qfrag[ks + 1][lane];
        dev::mma_f16(sa, a0, a1, a2, a3, qa.x, qa.y);
        dev::mma_f16(sb, a0, a1, a2, a3, qa.z, qa.w);
        dev::mma_f16(sc, b0, b1, b2, b3, qb.x, qb.y);
        dev::mma_f16(sd, b0, b1, b2, b3, qb.z, qb.w);
      }
      float sv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
        sv[r] = (sa[r] + sb[r]) + (sc[r] + sd[r]);
      // sv[0], sv[1]: key g, heads 2tq, 2tq+1; sv[2], sv[3]: key g + 8.
      if (int(g) >= nvalid)
        sv[0] = sv[1] = kNegInf;
      if (int(g) + 8 >= nvalid)
        sv[2] = sv[3] = kNegInf;
      float mx0 = fmaxf(sv[0], sv[2]), mx1 = fmaxf(sv[1], sv[3]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: key0 < len
      const float c0 = fast_exp(m0 - mn0), c1 = fast_exp(m1 - mn1);
      const float p0 = sv[0] == kNegInf ? 0.0f : fast_exp(sv[0] - mn0);
      const float p1 = sv[1] == kNegInf ? 0.0f : fast_exp(sv[1] - mn1);
      const float p2 = sv[2] == kNegInf ? 0.0f : fast_exp(sv[2] - mn0);
      const float p3 = sv[3] == kNegInf ? 0.0f : fast_exp(sv[3] - mn1);
      l0 = l0 * c0 + (p0 + p2);
      l1 = l1 * c1 + (p1 + p3);
      m0 = mn0, m1 = mn1;
#pragma unroll
      for (int mb = 0; mb < 16; ++mb)
        o[mb][0] *= c0, o[mb][1] *= c1, o[mb][2] *= c0, o[mb][3] *= c1;
      uint32_t h01, l01, h23, l23;
      dev::split_half2(p0, p1, h01, l01);
      dev::split_half2(p2, p3, h23, l23);
      const uint32_t bh0 = dev::movmatrix_t(h01), bh1 = dev::movmatrix_t(h23);
      const uint32_t bl0 = dev::movmatrix_t(l01), bl1 = dev::movmatrix_t(l23);
      // ---- O^T += V^T P^T ------------------------------------------------------------------
      const uint32_t vbase = dev::smem_u32(vst);
      const unsigned vrow = slab + (mi >> 1) * 8 + ri;
#pragma unroll
      for (int mb = 0; mb < 16; ++mb) {
        uint32_t a0, a1, a2, a3;
        dev::ldsm_x4_t(vbase + (mb >> 2) * kBoxBytes + dev::swz128(vrow, (mb & 3) * 2 + (mi & 1)),
                       a0, a1, a2, a3);
        dev::mma_f16(o[mb], a0, a1, a2, a3, bh0, bh1);
        dev::mma_f16(o[mb], a0, a1, a2, a3, bl0, bl1);
      }
    }
    __syncwarp();
    if (lane == 0)
      dev::mbar_arrive(dev::smem_u32(&sm.empty[k % kBars]));
  }
  if (cur_b != ~0u)
    finish(cur_b, cur_kvh);
  }  // t_begin < t_end
  }  // consumers
  __syncthreads();  // no thread exits while copies into this CTA's shared memory may be pending
}

}  // namespace miso::fast::decode
