#pragma once

// Causal gated GQA prefill on the 5th-generation tensor cores (tcgen05 + TMEM), the fast path
// behind miso_attn_prefill_tc().
//
// Work item (one CTA): 16 consecutive tokens x the 8 query heads of one KV head = 128 query rows
// (row r = token (r / 8), head (r % 8)), so every K / V tile is fetched once for all 8 heads that
// share it. Tiles are launched longest first (the causal triangle makes late tokens the most
// work), so the block scheduler approximates a longest-processing-time order.
//
// Per KV tile j of 128 keys:
//   S_j = Q K_j^T      tcgen05.mma M=128 N=128 K=256 (16 x K16; K arrives as two 128-dim halves),
//                      fp16 x fp16 -> fp32 in TMEM
//   softmax            8 warps, two per TMEM lane quadrant (one thread per row and half of the
//                      tile's columns; the pair exchanges row maxima through shared memory):
//                      causal mask on diagonal tiles only, online max (rescaling O only when
//                      the max grows by more than 2^8, then exactly), P = 2^(s - m) as fp16
//                      written into TMEM over the S tile it came from (two values per column)
//   O += P_j V_j       tcgen05.mma M=128 N=256 K=128 (8 x K16, V as two 64-key halves), A = P from
//                      TMEM, B = V (MN-major)
// With head dimension 256 a whole 128-key K or V tile (64 KB) does not fit twice next to Q, so K
// streams through a ring of 128-dim halves and V through a ring of 64-key halves (32 KB each);
// N = 128 for Q K^T runs at 97% of the tensor rate against 65% for N = 64.
// Roles: warps 0 and 2 issue TMA (Q and K halves, 3 slots; V halves, 2 slots), warp 1 owns TMEM
// and issues every MMA from one thread, warps 4-11 run softmax, O correction and the epilogue
// (O / l * sigmoid(gate), each warp staging its 32 rows through shared memory so global stores
// and gate loads are row-contiguous). Control decisions inside a softmax warp are warp-uniform
// (__all_sync), as the TMEM accesses are warp-collective.
//
// Precision: K / V are the fp16 cache, Q is fp16, P fp16 (bf16 P would cost ~1.6e-3 relative
// error), all accumulation fp32. Keys past pos0 + n are outside the K / V tensor maps and
// read as zeros, so garbage beyond the valid cache never reaches the MMAs.
//
// Every mbarrier wait is bounded; on a timeout the CTA records MISO_STATUS_TIMEOUT, stops issuing,
// drains the work it already issued (bounded) and frees its TMEM before exiting.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../common/device.cuh"
#include "../common/tcgen05.cuh"

namespace miso::fast::prefill {

constexpr int kQHeads = 16, kKvHeads = 2, kDim = 256, kGroup = 8;
constexpr int kTokens = 16;  // tokens per query tile; x 8 heads = 128 rows
constexpr int kRows = 128;
constexpr int kBN = 128;  // keys per KV tile
constexpr int kThreads = 384;  // warps 0 / 2 TMA, warp 1 MMA + TMEM, warps 4-11 softmax
constexpr uint32_t kQBox = kRows * 64 * 2;      // one 64-dim slab of Q: 16 KB
constexpr uint32_t kKBox = kBN * 64 * 2;        // one 64-dim slab of 128 keys: 16 KB
constexpr uint32_t kVBox = 64 * 64 * 2;         // one 64-dim slab of 64 keys: 8 KB
constexpr uint32_t kQBytes = 4 * kQBox;         // 64 KB
constexpr uint32_t kHalfBytes = 32768;          // a K half (2 slabs) or a V half (4 slabs)
constexpr int kKStages = 3, kVStages = 2;       // ring slots of K halves / V halves
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kQBytes;
constexpr uint32_t kOffV = kOffK + kKStages * kHalfBytes;
// Row-max exchange buffer: [2 parity][2 column half][128 rows] fp32.
constexpr uint32_t kOffRed = kOffV + kVStages * kHalfBytes;
constexpr uint32_t kOffBar = kOffRed + 2 * 2 * kRows * 4;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0;    // O accumulator: 256 columns
constexpr int kSBufs = 2;
// S buffers: kSBufs x 128 columns (P of the tile overwrites 64 of them).
constexpr uint32_t kColS = 256;

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kKStages], k_empty[kKStages], v_full[kVStages], v_empty[kVStages];
  uint64_t s_full[kSBufs], p_full[kSBufs], pv_done[2];
  uint64_t xchg[4][2];  // per TMEM lane quadrant and tile parity: the two softmax warps' partials
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t kSmemBytes = kOffBar + sizeof(Bars);  // base must be 1024-byte aligned
static_assert(2 * kKBox == kHalfBytes && 4 * kVBox == kHalfBytes, "ring slot size");
static_assert(kColS + kSBufs * kBN <= kTmemCols, "TMEM columns");
static_assert((kKStages + kVStages) * kHalfBytes >= kRows * kDim * 4,
              "O staging reuses the K and V stages");
static_assert(kSmemBytes <= 232448, "fits the 227 KB opt-in shared memory");

struct Args {
  const float* qg;
  float* core;
  unsigned pos0, n, qg_stride, n_qtiles;
};

__device__ __forceinline__ bool aborted(const Bars& b) {
  return *reinterpret_cast<const volatile int*>(&b.abort_flag) != 0;
}

// Bounded wait that also gives up at once if another role has aborted.
__device__ __forceinline__ bool wait_or_abort(Bars& b, uint64_t& bar, uint32_t parity) {
  if (aborted(b))
    return false;
  if (!dev::mbar_wait(dev::smem_u32(&bar), parity, 0x20)) {
    b.abort_flag = 1;
    return false;
  }
  return true;
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw;
  if ((dev::smem_u32(base) & 1023u) != 0) {  // the 128-byte swizzle needs 1024-byte alignment
    if (threadIdx.x == 0)
      dev::set_status(dev::kStatusTimeout);
    return;
  }
  Bars& bar = *reinterpret_cast<Bars*>(base + kOffBar);
  const unsigned warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const unsigned qt = a.n_qtiles - 1 - blockIdx.x / 2, kvh = blockIdx.x % 2;
  const unsigned t0 = qt * kTokens;
  const unsigned nq = min(static_cast<unsigned>(kTokens), a.n - t0);
  const unsigned key_end = a.pos0 + t0 + nq;  // keys [0, key_end) are seen by some row
  const unsigned nkv = (key_end + kBN - 1) / kBN;
  const uint32_t sbase = dev::smem_u32(base);

  if (threadIdx.x == 0) {
    dev::mbar_init(dev::smem_u32(&bar.q_full), 1);
    for (int s = 0; s < kKStages; ++s) {
      dev::mbar_init(dev::smem_u32(&bar.k_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.k_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      dev::mbar_init(dev::smem_u32(&bar.v_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.v_empty[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.pv_done[s]), 1);
      for (int qd = 0; qd < 4; ++qd)
        dev::mbar_init(dev::smem_u32(&bar.xchg[qd][s]), 2);
    }
    for (int s = 0; s < kSBufs; ++s) {
      dev::mbar_init(dev::smem_u32(&bar.s_full[s]), 1);
      dev::mbar_init(dev::smem_u32(&bar.p_full[s]), 8);
    }
    dev::mbar_init(dev::smem_u32(&bar.drain), 1);
    bar.abort_flag = 0;
    dev::mbar_init_fence();
  }
  if (warp == 1) {
    dev::tmem_alloc(dev::smem_u32(&bar.tmem_base), kTmemCols);
    dev::tmem_relinquish();
  }
  dev::tc_fence_before();
  __syncthreads();
  dev::tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------------------------ producers
    // Warp 0 loads Q and the K halves, warp 2 the V halves: the two rings refill independently
    // (half u of a ring as soon as the MMAs reading half u - slots have completed) and each
    // producer blocks in a suspending wait. Half u of K is dims [128 (u % 2), +128) of the 128
    // keys of tile u / 2; half u of V is keys [64 u, 64 u + 64) with all 256 dims.
    if (lane == 0) {
      const bool is_k = warp == 0;
      const CUtensorMap* map = is_k ? &kmap : &vmap;
      uint64_t* full = is_k ? bar.k_full : bar.v_full;
      uint64_t* empty = is_k ? bar.k_empty : bar.v_empty;
      const uint32_t dst0 = sbase + (is_k ? kOffK : kOffV);
      const unsigned nst = is_k ? kKStages : kVStages;
      dev::tma_prefetch_desc(map);
      if (is_k) {
        dev::tma_prefetch_desc(&qmap);
        dev::mbar_arrive_expect_tx(dev::smem_u32(&bar.q_full), kQBytes);
        for (int box = 0; box < 4; ++box)
          dev::tma_load_3d(sbase + kOffQ + box * kQBox, &qmap, box * 64, kvh * kGroup, t0,
                           dev::smem_u32(&bar.q_full));
      }
      unsigned issued = 0;
      for (unsigned u = 0; u < 2 * nkv; ++u) {
        const unsigned s = u % nst, ph = (u / nst) & 1;
        if (u >= nst && !wait_or_abort(bar, empty[s], ph ^ 1))
          break;
        const uint32_t fb = dev::smem_u32(&full[s]), dst = dst0 + s * kHalfBytes;
        dev::mbar_arrive_expect_tx(fb, kHalfBytes);
        if (is_k) {
          for (int box = 0; box < 2; ++box)
            dev::tma_load_3d(dst + box * kKBox, map, 128 * (u & 1) + 64 * box, (u >> 1) * kBN, kvh,
                             fb);
        } else {
          for (int box = 0; box < 4; ++box)
            dev::tma_load_3d(dst + box * kVBox, map, 64 * box, 64 * u, kvh, fb);
        }
        issued = u + 1;
      }
      if (aborted(bar)) {
        // Let the copies already issued land before the CTA exits (bounded waits).
        if (is_k)
          dev::mbar_wait(dev::smem_u32(&bar.q_full), 0);
        for (unsigned u = issued >= nst ? issued - nst : 0; u < issued; ++u)
          dev::mbar_wait(dev::smem_u32(&full[u % nst]), (u / nst) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t idesc_s = dev::idesc_f16_f32(kRows, kBN, 0, 0);
      const uint32_t idesc_o = dev::idesc_f16_f32(kRows, kDim, 0, 1);
      // Descriptors at offset 0; offsets are added to the start-address field.
      const uint64_t qdesc0 = dev::sdesc_sw128(sbase + kOffQ, 16, 1024);
      const uint64_t kdesc0 = dev::sdesc_sw128(sbase + kOffK, 16, 1024);
      const uint64_t vdesc0 = dev::sdesc_sw128(sbase + kOffV, kVBox, 1024);
      bool ok = wait_or_abort(bar, bar.q_full, 0);
      dev::tc_fence_after();
      // Issue state machine: S(j) goes out as soon as both K halves of tile j have landed and
      // PV(j - kSBufs) has been issued (S buffer j % kSBufs holds P_(j - kSBufs) until that PV has
      // read it; the tensor pipe runs in issue order); PV(i) as soon as P_i and both V halves of
      // tile i are ready. Both are polled, so a PV is never held back behind the next K load.
      unsigned ns = 0, np = 0;  // next S and next PV to issue
      long long last = clock64();
      while (ok && np < nkv) {
        bool progressed = false;
        if (ns < nkv && (ns < kSBufs || np + kSBufs > ns)) {
          const unsigned u0 = 2 * ns, s0 = u0 % kKStages, s1 = (u0 + 1) % kKStages;
          if (dev::mbar_test_wait(dev::smem_u32(&bar.k_full[s0]), (u0 / kKStages) & 1) &&
              dev::mbar_test_wait(dev::smem_u32(&bar.k_full[s1]), ((u0 + 1) / kKStages) & 1)) {
            dev::tc_fence_after();
            const uint32_t d = tmem + kColS + (ns % kSBufs) * kBN;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint64_t kd = kdesc0 + (((h ? s1 : s0) * kHalfBytes) >> 4);
#pragma unroll
              for (int ks = 0; ks < 8; ++ks)
                dev::tc_mma_f16_ss(
                    d, qdesc0 + ((((2 * h + (ks >> 2)) * kQBox) + (ks & 3) * 32) >> 4),
                    kd + (((ks >> 2) * kKBox + (ks & 3) * 32) >> 4), idesc_s, (h | ks) != 0);
              dev::tc_commit(dev::smem_u32(&bar.k_empty[h ? s1 : s0]));
            }
            dev::tc_commit(dev::smem_u32(&bar.s_full[ns % kSBufs]));
            ++ns;
            progressed = true;
          }
        }
        if (np < ns) {
          const unsigned i = np, sb = i % kSBufs, sph = (i / kSBufs) & 1;
          // V halves 2i and 2i + 1 sit in slots 0 and 1 (two slots), phase i & 1.
          if (dev::mbar_test_wait(dev::smem_u32(&bar.p_full[sb]), sph) &&
              dev::mbar_test_wait(dev::smem_u32(&bar.v_full[0]), i & 1) &&
              dev::mbar_test_wait(dev::smem_u32(&bar.v_full[1]), i & 1)) {
            dev::tc_fence_after();
            const uint32_t pa = tmem + kColS + sb * kBN;  // P_i: 128 keys as 64 fp16 pairs
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint64_t vd = vdesc0 + ((h * kHalfBytes) >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                dev::tc_mma_f16_ts(tmem + kColO, pa + 32 * h + 8 * kk, vd + ((kk * 2048) >> 4),
                                   idesc_o, (i > 0 || h > 0 || kk > 0) ? 1u : 0u);
              dev::tc_commit(dev::smem_u32(&bar.v_empty[h]));
            }
            dev::tc_commit(dev::smem_u32(&bar.pv_done[i & 1]));
            ++np;
            progressed = true;
          }
        }
        if (progressed) {
          last = clock64();
        } else if (aborted(bar)) {
          ok = false;
        } else if (clock64() - last > dev::kWaitLimitCycles) {  // nothing became ready: give up
          dev::set_status(dev::kStatusTimeout, 0x21);
          bar.abort_flag = 1;
          ok = false;
        } else {
          __nanosleep(20);  // short: this thread is on the critical path, but shares issue slots
        }
      }
      // Every MMA issued above has completed once `drain` flips (bounded).
      dev::tc_commit(dev::smem_u32(&bar.drain));
      dev::mbar_wait(dev::smem_u32(&bar.drain), 0);
    }
  } else if (warp >= 4) {
    // --------------------------------------------------------------- softmax and epilogue
    // Two warps per TMEM lane quadrant: warp (4 + q + 4 hc) holds rows [32 q, 32 q + 32) and
    // S columns [64 hc, 64 hc + 64) of each tile, O columns [128 hc, 128 hc + 128).
    const unsigned q = warp & 3, hc = (warp - 4) >> 2;
    const unsigned r = 32 * q + lane;
    const uint32_t trow = tmem + ((32u * q) << 16);
    const unsigned tok = t0 + r / kGroup;
    const unsigned pos = a.pos0 + tok;        // this row sees keys [0, pos]
    const unsigned pos_min = a.pos0 + t0;     // no row of the tile sees fewer keys
    float* red = reinterpret_cast<float*>(base + kOffRed);
    const float sl2 = 1.4426950408889634f * 0.0625f;  // log2(e) / sqrt(256)
    const float kNegInf = -__int_as_float(0x7f800000);
    float m_ref = kNegInf, l = 0.0f;
    bool ok = true;
    {
      // The epilogue's gate rows (this warp's 32 rows, 512 bytes each) into L2 now, so that the
      // epilogue finds them there: lane = row, four 128-byte lines each.
      const unsigned rr = 32 * q + lane, tk = t0 + rr / kGroup;
      if (tk < a.n) {
        const float* g = a.qg + size_t(tk) * a.qg_stride + (kvh * kGroup + rr % kGroup) * 2 * kDim +
                         kDim + 128 * hc;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(g + 32 * e));
      }
    }
    // Exchange of one float per row with the partner warp through red[] and an mbarrier with
    // one arrival per warp (bounded wait); returns the partner's value.
    auto exchange = [&](unsigned j, float mine, float& theirs) -> bool {
      red[((j & 1) * 2 + hc) * kRows + r] = mine;
      __syncwarp();
      if (lane == 0)
        dev::mbar_arrive(dev::smem_u32(&bar.xchg[q][j & 1]));
      if (!__all_sync(0xffffffffu, wait_or_abort(bar, bar.xchg[q][j & 1], (j >> 1) & 1)))
        return false;
      theirs = red[((j & 1) * 2 + (1 - hc)) * kRows + r];
      return true;
    };
    for (unsigned j = 0; j < nkv; ++j) {
      const unsigned s = j % kSBufs, ph = (j / kSBufs) & 1;  // S / P buffer of tile j
      if (!__all_sync(0xffffffffu, wait_or_abort(bar, bar.s_full[s], ph))) {
        ok = false;
        break;
      }
      dev::tc_fence_after();
      float v[64];
      dev::tmem_ld32(trow + kColS + s * kBN + 64 * hc, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      dev::tmem_ld32(trow + kColS + s * kBN + 64 * hc + 32,
                     *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      dev::tmem_wait_ld();
      // Raw scores (the scale is folded into the exponent's FMA below; it is positive, so the
      // maximum commutes with it). Four partial maxima keep the dependency chain short.
      const unsigned key0 = j * kBN + 64 * hc;
      float mx4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
      if (key0 + 63 <= pos_min) {  // interior tile half: no masking
#pragma unroll
        for (int c = 0; c < 64; ++c)
          mx4[c & 3] = fmaxf(mx4[c & 3], v[c]);
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          v[c] = key0 + c <= pos ? v[c] : kNegInf;
          mx4[c & 3] = fmaxf(mx4[c & 3], v[c]);
        }
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      float mx_other;
      if (!exchange(j, mx, mx_other)) {
        ok = false;
        break;
      }
      const float m_new = fmaxf(m_ref, fmaxf(mx, mx_other) * sl2);
      if (j == 0) {
        m_ref = m_new;  // O is written (not accumulated) by the first P V
      } else if (__any_sync(0xffffffffu, m_new > m_ref + 8.0f)) {
        // Both warps of the pair see the same rows and maxima, so they take this branch
        // together; each rescales its 128 O columns once PV_{j-1} has landed.
        const unsigned i = j - 1;
        if (!__all_sync(0xffffffffu, wait_or_abort(bar, bar.pv_done[i & 1], (i >> 1) & 1))) {
          ok = false;
          break;
        }
        dev::tc_fence_after();
        const float corr = dev::ex2_approx(m_ref - m_new);
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t o[32];
          dev::tmem_ld32(trow + kColO + 128 * hc + ch * 32, o);
          dev::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e)
            o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
          dev::tmem_st32(trow + kColO + 128 * hc + ch * 32, o);
        }
        dev::tmem_wait_st();
        l *= corr;
        m_ref = m_new;
      }
      // P overwrites this warp's half of P's 64 columns in the S buffer: both warps of the pair
      // have read their S halves before the exchange above, so nothing unread is overwritten.
      const float neg_m = -m_ref;
      float lsum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint32_t pk[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float p0 = dev::ex2_approx(fmaf(v[2 * e], sl2, neg_m));
        const float p1 = dev::ex2_approx(fmaf(v[2 * e + 1], sl2, neg_m));
        const __half2 h2v = __floats2half2_rn(p0, p1);
        pk[e] = *reinterpret_cast<const uint32_t*>(&h2v);
        lsum[e & 3] += p0 + p1;
      }
      dev::tmem_st32(trow + kColS + s * kBN + 32 * hc, pk);
      l += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
      dev::tmem_wait_st();
      dev::tc_fence_before();
      __syncwarp();
      if (lane == 0)
        dev::mbar_arrive(dev::smem_u32(&bar.p_full[s]));
    }
    // ---- epilogue: core = O / l * sigmoid(gate), staged through the (now idle) K/V stages ----
    const unsigned last = nkv - 1;
    float l_other = 0.0f;
    if (ok && exchange(nkv, l, l_other) &&
        __all_sync(0xffffffffu, wait_or_abort(bar, bar.pv_done[last & 1], (last >> 1) & 1))) {
      dev::tc_fence_after();
      // This warp's 32 rows x 128 columns, float4 index XOR-swizzled by row % 8.
      float* stage = reinterpret_cast<float*>(base + kOffK) + (warp - 4) * 32 * 128;
      const float inv_l = 1.0f / (l + l_other);
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t o[32];
        dev::tmem_ld32(trow + kColO + 128 * hc + ch * 32, o);
        dev::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const unsigned phys = (ch * 8 + i) ^ (lane & 7);
          reinterpret_cast<float4*>(stage + lane * 128)[phys] =
              make_float4(__uint_as_float(o[4 * i]) * inv_l, __uint_as_float(o[4 * i + 1]) * inv_l,
                          __uint_as_float(o[4 * i + 2]) * inv_l,
                          __uint_as_float(o[4 * i + 3]) * inv_l);
        }
      }
      __syncwarp();
      // Rows in groups of 8 (one token, its 8 heads): the group's gate loads are all issued
      // before any is used, so a warp waits for 4 memory round trips instead of 32.
#pragma unroll 1
      for (unsigned lr0 = 0; lr0 < 32; lr0 += kGroup) {
        const unsigned tk = t0 + (32 * q + lr0) / kGroup;
        if (tk >= a.n)
          break;
        const float* grow = a.qg + size_t(tk) * a.qg_stride + kDim + 128 * hc;
        float4 g[kGroup];
#pragma unroll
        for (int e = 0; e < kGroup; ++e)
          g[e] = reinterpret_cast<const float4*>(grow + (kvh * kGroup + e) * 2 * kDim)[lane];
#pragma unroll
        for (int e = 0; e < kGroup; ++e) {
          const unsigned lr = lr0 + e, h = kvh * kGroup + e;
          const float4 ov = reinterpret_cast<const float4*>(stage + lr * 128)[lane ^ (lr & 7)];
          reinterpret_cast<float4*>(a.core + (size_t(tk) * kQHeads + h) * kDim + 128 * hc)[lane] =
              make_float4(ov.x / (1.0f + __expf(-g[e].x)), ov.y / (1.0f + __expf(-g[e].y)),
                          ov.z / (1.0f + __expf(-g[e].z)), ov.w / (1.0f + __expf(-g[e].w)));
        }
      }
    }
  }

  dev::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    dev::tc_fence_after();
    dev::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace miso::fast::prefill
