#pragma once

// Batched Gated DeltaNet decode step: the per-token arithmetic of deltanet_step_op
// (kernels/deltanet_step.hpp) for `batch` independent sequences in one launch, the fast path
// behind miso_deltanet_step_batched().
//
// The step reads and writes every sequence's 32 x 128 x 128 fp32 state once (128 KB per
// (sequence, head) of traffic, 268 MB per step at batch 64), so it is HBM-bound. A persistent
// kernel, two 512-thread CTAs per SM, walks the (sequence, head) units. A unit's 64 KB state
// arrives by a TMA load (four [128 k][32 v] boxes, 128-byte swizzled), its conv inputs and gate
// by bulk copies into one of two input stages. As soon as every warp has read the state into
// registers (an mbarrier with one arrival per warp), the next unit's copies are issued, so they
// are in flight for the whole of this unit's computation.
//
// Thread layout: warp w owns the value columns [8 w, 8 w + 8) over all 128 key rows; lane l holds
// rows (l % 16) + 16 j (j = 0..7) of columns 8 w + 4 (l / 16) + [0, 4). The sums over k
// (S^T k and S^T q) are then warp shuffles; a unit needs two CTA barriers (the conv outputs, the
// gated norm's sum over all 128 columns). The updated state goes from registers to global memory,
// lanes l and l + 16 writing the two halves of a row's 32-byte segment.

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>

#include "../common/device.cuh"
#include "../kernels/deltanet_step.hpp"

namespace miso::fast::dnstep {

constexpr int kDim = 128, kKHeads = 16, kVHeads = 32, kCh = 8192;
constexpr int kWarps = 16, kThreads = kWarps * 32;
constexpr int kCtasPerSm = 2;

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

// Dynamic shared memory (base rounded up to 1024 bytes for the swizzled boxes):
//   [0, 64K)        state: box x (v columns [32 x, +32)) at 16K x, [128 rows k][128 B] swizzled
//   then            two input stages (units alternate): x [384] of the unit's conv channels (q, k,
//                   v in that order), their history [384][3] and conv_w [384][4]; z [128]; the
//                   sequence's a and b rows [32] each
//   then            conv outputs q, k, v [128] each, SiLU(z) [128], ssm_a and dt_bias [32] each,
//                   the q / k sums of squares [8], the norm partials [2][16], the mbarriers
constexpr uint32_t kStateBytes = kDim * kDim * 4;
constexpr uint32_t kInX = 0, kInHist = 384 * 4, kInW = kInHist + 384 * 12, kInZ = kInW + 384 * 16;
constexpr uint32_t kInA = kInZ + kDim * 4, kInB = kInA + kVHeads * 4;
constexpr uint32_t kInBytes = kInB + kVHeads * 4;
constexpr uint32_t kOffIn = kStateBytes, kOffQ = kOffIn + 2 * kInBytes;
constexpr uint32_t kOffK = kOffQ + kDim * 4, kOffV = kOffK + kDim * 4;
constexpr uint32_t kOffG = kOffV + kDim * 4, kOffSa = kOffG + kDim * 4, kOffDt = kOffSa + 128;
constexpr uint32_t kOffNrm = kOffDt + 128, kOffRed = kOffNrm + 32;
constexpr uint32_t kOffBar = kOffRed + 2 * kWarps * 4;  // full_s, empty_s, full_in[2]
constexpr size_t kSmemBytes = kOffBar + 4 * 8 + 1024;
static_assert(kInBytes % 16 == 0 && kOffBar % 8 == 0, "bulk copy / mbarrier alignment");
static_assert(kCtasPerSm * kSmemBytes <= 228 * 1024, "two CTAs per SM");

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// Channel of local conv channel i (0..383: q, k, v of the unit's heads).
__device__ __forceinline__ unsigned conv_channel(unsigned i, unsigned kh, unsigned h) {
  const unsigned which = i / kDim, ii = i % kDim;
  return which == 0 ? kh * kDim + ii
       : which == 1 ? kKHeads * kDim + kh * kDim + ii
                    : 2 * kKHeads * kDim + h * kDim + ii;
}

// Copies of unit u: its state (four swizzled boxes) on `bar`. One thread.
__device__ __forceinline__ void issue_state(const CUtensorMap* smap, unsigned u, uint32_t sbase,
                                            uint32_t bar) {
  dev::mbar_arrive_expect_tx(bar, kStateBytes);
#pragma unroll
  for (int x = 0; x < 4; ++x)
    dev::tma_load_2d(sbase + x * 16384, smap, 32 * x, int(u * kDim), bar);
}

// Copies of unit u: its conv inputs and z into the input stage at `dst` on `bar`. One thread.
__device__ __forceinline__ void issue_inputs(const Args& p, unsigned u, uint32_t dst,
                                             uint32_t bar) {
  const unsigned bq = u / kVHeads, h = u % kVHeads, kh = h % kKHeads;
  dev::mbar_arrive_expect_tx(bar, kInBytes);
  const unsigned c0[3] = {kh * kDim, kKHeads * kDim + kh * kDim, 2 * kKHeads * kDim + h * kDim};
#pragma unroll
  for (int g = 0; g < 3; ++g) {
    dev::bulk_load(dst + kInX + g * 512, p.qkv + size_t(bq) * p.in_stride + c0[g], 512, bar);
    dev::bulk_load(dst + kInHist + g * 1536, p.conv_in + (size_t(bq) * kCh + c0[g]) * 3, 1536,
                   bar);
    dev::bulk_load(dst + kInW + g * 2048, p.conv_w + size_t(c0[g]) * 4, 2048, bar);
  }
  dev::bulk_load(dst + kInZ, p.z + size_t(bq) * p.in_stride + h * kDim, 512, bar);
  dev::bulk_load(dst + kInA, p.a + size_t(bq) * p.in_stride, kVHeads * 4, bar);
  dev::bulk_load(dst + kInB, p.b + size_t(bq) * p.in_stride, kVHeads * 4, bar);
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    step_batched_kernel(const __grid_constant__ CUtensorMap smap, Args p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = dev::smem_u32(smem_raw), sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  float* qs = reinterpret_cast<float*>(smem + kOffQ);
  float* ks = reinterpret_cast<float*>(smem + kOffK);
  float* vs = reinterpret_cast<float*>(smem + kOffV);
  float* gs = reinterpret_cast<float*>(smem + kOffG);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* nrm = reinterpret_cast<float*>(smem + kOffNrm);
  float* sas = reinterpret_cast<float*>(smem + kOffSa);
  float* dts = reinterpret_cast<float*>(smem + kOffDt);
  const uint32_t full_s = sbase + kOffBar, empty_s = full_s + 8, full_in0 = full_s + 16;

  const unsigned t = threadIdx.x, w = t / 32, lane = t % 32;
  const unsigned hl = lane / 16, rl = lane % 16;   // column half, row lane
  const unsigned units = p.batch * kVHeads, G = gridDim.x;
  const unsigned n_local = blockIdx.x < units ? (units - blockIdx.x + G - 1) / G : 0;
  if (t == 0) {
    dev::mbar_init(full_s, 1);
    dev::mbar_init(empty_s, kWarps);
    dev::mbar_init(full_in0, 1);
    dev::mbar_init(full_in0 + 8, 1);
    dev::mbar_init_fence();
    dev::tma_prefetch_desc(&smap);
  }
  if (t < kVHeads) {
    sas[t] = p.ssm_a[t];
    dts[t] = p.dt_bias[t];
  }
  __syncthreads();
  if (t == 0 && n_local > 0) {
    issue_inputs(p, blockIdx.x, sbase + kOffIn, full_in0);
    issue_state(&smap, blockIdx.x, sbase, full_s);
  }
  // The state float4 of row r: box w / 4, 16-byte chunk 2 (w % 4) + hl, XOR-swizzled by r % 8.
  const uint32_t chunk = 2 * (w % 4) + hl;
  const uint8_t* sbox = smem + (w / 4) * 16384;
  const unsigned col0 = 8 * w + 4 * hl;            // first of the thread's four columns
  const unsigned my_e = (lane >> 2) & 3;           // column (of the half) the reductions leave here
  unsigned aborted_at = n_local;  // the unit at which a timed-out wait ended the walk
  bool issued = false;            // (thread 0) the copies of unit i + 1 were issued in unit i

  for (unsigned i = 0; i < n_local; ++i) {
    const unsigned u = blockIdx.x + i * G, bq = u / kVHeads, h = u % kVHeads;
    const unsigned kh = h % kKHeads, st = i & 1;
    const uint8_t* in = smem + kOffIn + st * kInBytes;
    bool got = dev::mbar_wait(full_s, i & 1, 0x14);
    float4 s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const unsigned r = rl + 16 * j;
      s[j] = *reinterpret_cast<const float4*>(sbox + r * 128 + ((chunk ^ (r & 7)) << 4));
    }
    // The state is in registers: once every warp has read it, thread 0 refills the stage with
    // the next unit's state and the other input stage with the next unit's inputs.
    dev::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0)
      dev::mbar_arrive(empty_s);
    issued = false;
    if (t == 0 && got && i + 1 < n_local) {
      if (dev::mbar_wait(empty_s, i & 1, 0x14)) {
        issued = true;
        issue_state(&smap, u + G, sbase, full_s);
        issue_inputs(p, u + G, sbase + kOffIn + (st ^ 1) * kInBytes, full_in0 + 8 * (st ^ 1));
      } else {
        got = false;
      }
    }
    got = __all_sync(0xffffffffu, dev::mbar_wait(full_in0 + 8 * st, (i >> 1) & 1, 0x14) && got);
    // Conv + SiLU of the unit's 384 channels (thread t < 384: channel t), the gate SiLU(z).
    if (got && t < 3 * kDim) {
      const float4 cw = reinterpret_cast<const float4*>(in + kInW)[t];
      const float* hi = reinterpret_cast<const float*>(in + kInHist) + 3 * t;
      const float x = reinterpret_cast<const float*>(in + kInX)[t];
      const float y = silu(cw.x * hi[0] + cw.y * hi[1] + cw.z * hi[2] + cw.w * x);
      if (t >= 2 * kDim || h < kKHeads) {
        float* co = p.conv_out + (size_t(bq) * kCh + conv_channel(t, kh, h)) * 3;
        co[0] = hi[1];
        co[1] = hi[2];
        co[2] = x;
      }
      (t < kDim ? qs : t < 2 * kDim ? ks : vs)[t % kDim] = y;
      if (t < 2 * kDim) {  // sums of squares of q (warps 0-3) and k (warps 4-7)
        const float ss = miso::kernels::wave_sum(y * y);
        if (lane == 0)
          nrm[w] = ss;
      }
    } else if (got) {
      gs[t - 3 * kDim] = silu(reinterpret_cast<const float*>(in + kInZ)[t - 3 * kDim]);
    }
    // (A) conv outputs visible. A timed-out wait in any thread ends the CTA's walk here, before
    // the unit writes its state or outputs (the status word records it).
    if (__syncthreads_or(!got)) {
      aborted_at = i;
      break;
    }

    const float* ins = reinterpret_cast<const float*>(in);
    const float beta = 1.0f / (1.0f + __expf(-ins[(kInB >> 2) + h]));
    const float decay = __expf(
        sas[h] * miso::kernels::deltanet_detail::softplus(ins[(kInA >> 2) + h] + dts[h]));
    // L2 norms of q and k.
    const float qscale = rsqrtf(nrm[0] + nrm[1] + nrm[2] + nrm[3] + 1e-6f) *
                         rsqrtf(static_cast<float>(kDim));
    const float kscale = rsqrtf(nrm[4] + nrm[5] + nrm[6] + nrm[7] + 1e-6f);

    // S = decay S; S^T k over the thread's rows, then summed over the 16 row lanes: a
    // reduce-scatter leaves column my_e of the half in each lane (4 lanes per column).
    float p4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float kk = ks[rl + 16 * j] * kscale;
      s[j].x *= decay, s[j].y *= decay, s[j].z *= decay, s[j].w *= decay;
      p4[0] += s[j].x * kk, p4[1] += s[j].y * kk, p4[2] += s[j].z * kk, p4[3] += s[j].w * kk;
    }
    auto reduce_scatter = [&](const float (&v)[4]) {
      const bool b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
      const float r0 = (b3 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, b3 ? v[0] : v[2], 8);
      const float r1 = (b3 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, b3 ? v[1] : v[3], 8);
      float r = (b2 ? r1 : r0) + __shfl_xor_sync(0xffffffffu, b2 ? r0 : r1, 4);
      r += __shfl_xor_sync(0xffffffffu, r, 2);
      r += __shfl_xor_sync(0xffffffffu, r, 1);
      return r;
    };
    const float kvs = reduce_scatter(p4);
    const float dm = (vs[col0 + my_e] - kvs) * beta;  // delta of column col0 + my_e
    float d[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      d[e] = __shfl_sync(0xffffffffu, dm, (lane & 16) | (e << 2));
    // S += k delta^T; o = S^T q; the new state to global memory.
    float4* S = reinterpret_cast<float4*>(p.state + size_t(u) * kDim * kDim + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float kk = ks[rl + 16 * j] * kscale, qq = qs[rl + 16 * j] * qscale;
      s[j].x += kk * d[0], s[j].y += kk * d[1], s[j].z += kk * d[2], s[j].w += kk * d[3];
      p4[0] = (j ? p4[0] : 0.0f) + s[j].x * qq;
      p4[1] = (j ? p4[1] : 0.0f) + s[j].y * qq;
      p4[2] = (j ? p4[2] : 0.0f) + s[j].z * qq;
      p4[3] = (j ? p4[3] : 0.0f) + s[j].w * qq;
      S[size_t(rl + 16 * j) * (kDim / 4)] = s[j];
    }
    const float o = reduce_scatter(p4);  // o of column col0 + my_e
    // Gated RMS norm over the 128 columns (each column is held by 4 lanes).
    float so = o * o;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      so += __shfl_xor_sync(0xffffffffu, so, off);
    if (lane == 0)
      red[(i & 1) * kWarps + w] = 0.25f * so;
    const unsigned v = col0 + my_e;
    const float gate = p.norm_w[v] * gs[v];  // read before (B): the next unit rewrites gs
    __syncthreads();  // (B)
    float tot = 0.0f;
#pragma unroll
    for (int r = 0; r < kWarps; ++r)
      tot += red[(i & 1) * kWarps + r];
    if ((lane & 3) == 0) {
      const float rr = rsqrtf(tot / kDim + p.eps);
      p.out[size_t(bq) * kVHeads * kDim + h * kDim + v] = o * rr * gate;
    }
  }
  // No thread leaves while a copy into this CTA's shared memory may still be landing (after a
  // timed-out wait): thread 0 waits (bounded) for the copies of the unit where the walk ended and,
  // if they were issued, of the next one (a phase that already completed passes at once).
  if (t == 0 && aborted_at < n_local)
    for (unsigned k = aborted_at; k <= aborted_at + (issued ? 1u : 0u); ++k) {
      dev::mbar_wait(full_s, k & 1);
      dev::mbar_wait(full_in0 + 8 * (k & 1), (k >> 1) & 1);
    }
  __syncthreads();
}

}  // namespace miso::fast::dnstep
