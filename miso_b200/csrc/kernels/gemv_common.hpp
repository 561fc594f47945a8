#pragma once

// Row-dot machinery shared by the quantised decode GEMVs (q4k_gemv.hpp, q6k_gemv.hpp,
// mixed_gemv.hpp) and the decode MoE kernels, for the two weight layouts the reference engine
// uploads (src/repack.hpp:14-31):
//   Q4_K r1: GGUF Q4_K blocks of 256 weights (d, dmin, 12 scale bytes, 128 nibble bytes) whose
//            bytes 4..15 are rewritten so nibble group g holds sc[2g] | m[2g] << 6 |
//            sc[2g+1] << 12 | m[2g+1] << 18 as 24 little-endian bits at byte 4 + 3g;
//            weight = d * sc * q - dmin * m.
//   Q6_K r1: a row of nb blocks stored as sections [ql nb*128][qh nb*64][scales nb*16][d nb*2],
//            padded to a multiple of 16 bytes; weight = d * scale * (q - 32), q 6 bits.
// Activations are converted once, when a block stages them (FP16 rounding, or the per-32 absmax
// INT8 format), and every product is accumulated in FP32.
//
// Work unit: a "chunk" is one 16-byte load of a row's low-bit bytes = 32 weights (16 of them from
// the low nibbles, 16 from the high nibbles). A lane takes chunks lane, lane + 32, ... of a row,
// so a warp's loads are contiguous. The activations a chunk needs are the same for every row, so a
// block stages them once in shared memory in chunk order ([8 float4][chunks]: float4 v of chunk c
// at v * chunks + c), which makes the per-row reads conflict-free; the per-16 sums of the rounded
// activations (the dmin * m term of Q4_K) are staged beside them.

#include <cuda_fp16.h>

#include <cstddef>
#include <cstdint>

#include "wave.hpp"

namespace miso::kernels {

namespace gemv {

// x rounded to binary16 and back (round to nearest even), the activation format of the GEMVs.
__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

// An integer 0 <= v < 2^23 as a float, exactly, without an integer-to-float conversion: the bits
// 0x4B000000 | v are the float 2^23 + v.
__device__ __forceinline__ float small_int_f(uint32_t v) {
  return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}

// A 6-bit code q as the float q - 32, exactly (one add, as above).
__device__ __forceinline__ float q6_f(uint32_t q) {
  return __uint_as_float(0x4B000000u | q) - 8388640.0f;
}

__device__ __forceinline__ float f16_bits(uint32_t h) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

enum class Fmt { Q4K, Q6K };

__host__ __device__ constexpr std::size_t q4k_row_bytes(unsigned k) { return std::size_t{k} / 256 * 144; }
__host__ __device__ constexpr std::size_t q6k_row_bytes(unsigned k) {
  return (std::size_t{k} / 256 * 210 + 15) / 16 * 16;
}
template <Fmt F>
__host__ __device__ constexpr std::size_t row_bytes(unsigned k) {
  return F == Fmt::Q4K ? q4k_row_bytes(k) : q6k_row_bytes(k);
}

// Position, within the K activations, of element i (0..15) of half `hi` (0 = the weights from low
// nibbles, 1 = high nibbles) of chunk c.
template <Fmt F>
__host__ __device__ constexpr unsigned chunk_elem(unsigned c, unsigned hi, unsigned i) {
  if (F == Fmt::Q4K) {
    // Chunk j = c % 8 of block c / 8 is bytes 16 j.. of the 128 nibble bytes: group g = j / 2
    // (bytes 32 g..32 g + 31), half h = j % 2. Low nibbles are sub-block 2g, high 2g + 1.
    const unsigned b = c / 8, j = c % 8;
    return 256 * b + 64 * (j / 2) + 32 * hi + 16 * (j % 2) + i;
  } else {
    // Chunk j = c % 8 of block c / 8 is ql bytes 16 j..: half n = j / 4, quarter p = j % 4.
    // ql bytes 64n + l (l < 32) carry elements 128n + l (low nibble) and 128n + 64 + l (high);
    // bytes 64n + 32 + l carry 128n + 32 + l and 128n + 96 + l.
    const unsigned b = c / 8, j = c % 8, n = j / 4, p = j % 4;
    return 256 * b + 128 * n + 64 * hi + 32 * (p / 2) + 16 * (p % 2) + i;
  }
}

// Inverse of chunk_elem: element e -> (chunk, half, i).
template <Fmt F>
__host__ __device__ constexpr void elem_chunk(unsigned e, unsigned& c, unsigned& hi, unsigned& i) {
  const unsigned b = e / 256, r = e % 256;
  if (F == Fmt::Q4K) {
    const unsigned g = r / 64, s = r % 64;
    hi = s / 32, i = s % 16;
    c = 8 * b + 2 * g + (s % 32) / 16;
  } else {
    const unsigned n = r / 128, s = r % 128;
    hi = s / 64, i = s % 16;
    const unsigned l = s % 64;  // 32 (p / 2) + 16 (p % 2) + i
    c = 8 * b + 4 * n + 2 * (l / 32) + (l % 32) / 16;
  }
}

// Activation formats (the reference's ActFormat, kernels/q4k_gemv.hpp:18-21): FP16-rounded
// values, or per-32 absmax INT8 (x = q * amax / 127, q = rint(x * 127 / amax), |q| <= 127), both
// applied once when the activations are staged and multiplied in FP32.
enum class Act { Fp16, Int8 };

// Shared-memory activations for K elements: xv[8][K / 32] float4 (chunk order), sums[2][K / 32]
// of each half chunk, and one INT8 scale per 32 consecutive elements.
template <unsigned K>
struct StagedX {
  static constexpr unsigned kChunks = K / 32;
  float4 xv[8 * kChunks];
  float sum[2 * kChunks];
  float scale[K / 32];
};

// Stages x (K floats, global or shared) into `s` in F's chunk order, converted to format A. All
// threads of the block take part; ends with a barrier.
template <Fmt F, unsigned K, int kBlock, Act A = Act::Fp16>
__device__ inline void stage_x(const float* x, StagedX<K>& s) {
  constexpr unsigned kChunks = K / 32;
  if (A == Act::Int8) {
    for (unsigned q = threadIdx.x; q < K / 32; q += kBlock) {
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i)
        amax = fmaxf(amax, fabsf(x[32 * q + i]));
      s.scale[q] = amax;
    }
    __syncthreads();
  }
  float* xs = reinterpret_cast<float*>(s.xv);
  for (unsigned e = threadIdx.x; e < K; e += kBlock) {
    unsigned c, hi, i;
    elem_chunk<F>(e, c, hi, i);
    const unsigned v = 4 * hi + i / 4;
    float xe;
    if (A == Act::Int8) {
      const float amax = s.scale[e / 32];
      xe = amax > 0.0f ? rintf(x[e] * 127.0f / amax) * (amax / 127.0f) : 0.0f;
    } else {
      xe = round_f16(x[e]);
    }
    xs[(v * kChunks + c) * 4 + i % 4] = xe;
  }
  __syncthreads();
  for (unsigned q = threadIdx.x; q < 2 * kChunks; q += kBlock) {
    const unsigned hi = q / kChunks, c = q % kChunks;
    float acc = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const float4 f = s.xv[(4 * hi + v) * kChunks + c];
      acc += f.x + f.y + f.z + f.w;
    }
    s.sum[hi * kChunks + c] = acc;
  }
  __syncthreads();
}

// The bytes of one chunk of one row.
struct ChunkW {
  uint4 lo;   // Q4_K: the 16 nibble bytes; Q6_K: the 16 ql bytes
  uint4 aux;  // Q4_K: the block's 16-byte header; Q6_K: the 16 qh bytes carrying the top bits
  uint32_t sd;  // Q6_K: the two int8 scales (bytes 0, 1) and d (bits 16..31); unused for Q4_K
};

template <Fmt F>
__device__ __forceinline__ ChunkW load_chunk(const uint8_t* row, unsigned k, unsigned c) {
  ChunkW w;
  const unsigned b = c / 8, j = c % 8;
  if (F == Fmt::Q4K) {
    const uint8_t* blk = row + std::size_t{b} * 144;
    w.lo = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * j));
    w.aux = __ldg(reinterpret_cast<const uint4*>(blk));
    w.sd = 0;
  } else {
    const unsigned nb = k / 256, n = j / 4, p = j % 4;
    w.lo = __ldg(reinterpret_cast<const uint4*>(row + std::size_t{b} * 128 + 16 * j));
    w.aux = __ldg(reinterpret_cast<const uint4*>(row + std::size_t{nb} * 128 + b * 64 + 32 * n +
                                                 16 * (p % 2)));
    // Scales of this chunk: group l / 16 = p % 2 of quarter u, u = p / 2 (low) and p / 2 + 2 (high):
    // index 8n + (p % 2) + 2u.
    const int8_t* sc = reinterpret_cast<const int8_t*>(row + std::size_t{nb} * 192 + b * 16);
    const int s_lo = sc[8 * n + (p % 2) + 2 * (p / 2)];
    const int s_hi = sc[8 * n + (p % 2) + 2 * (p / 2 + 2)];
    const uint32_t d = *reinterpret_cast<const uint16_t*>(row + std::size_t{nb} * 208 + b * 2);
    w.sd = (static_cast<uint32_t>(s_lo) & 0xFFu) | (static_cast<uint32_t>(s_hi) & 0xFFu) << 8 |
           d << 16;
  }
  return w;
}

// 32-bit word `i` (0..3) of a uint4.
__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Contribution of one chunk of one row against staged activations.
template <Fmt F, unsigned K>
__device__ __forceinline__ float chunk_dot(const ChunkW& w, const StagedX<K>& s, unsigned c) {
  constexpr unsigned kChunks = K / 32;
  float acc_lo = 0.0f, acc_hi = 0.0f;
  if (F == Fmt::Q4K) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint32_t q = word(w.lo, v);
      const float4 xl = s.xv[v * kChunks + c], xh = s.xv[(4 + v) * kChunks + c];
      acc_lo += small_int_f(q & 15u) * xl.x + small_int_f((q >> 8) & 15u) * xl.y +
                small_int_f((q >> 16) & 15u) * xl.z + small_int_f((q >> 24) & 15u) * xl.w;
      acc_hi += small_int_f((q >> 4) & 15u) * xh.x + small_int_f((q >> 12) & 15u) * xh.y +
                small_int_f((q >> 20) & 15u) * xh.z + small_int_f(q >> 28) * xh.w;
    }
    // Header: d (bits 0..15 of word 0), dmin (16..31); the 24-bit field of group g starts at
    // bit 32 + 24 g.
    const unsigned g = (c % 8) / 2, bit = 24 * g;
    const uint32_t lo_w = word(w.aux, 1 + bit / 32);
    const uint32_t hi_w = bit / 32 + 2 < 4 ? word(w.aux, 2 + bit / 32) : 0u;
    const uint32_t f = __funnelshift_r(lo_w, hi_w, bit % 32);
    const float d = f16_bits(w.aux.x & 0xFFFFu), dmin = f16_bits(w.aux.x >> 16);
    const float sc0 = small_int_f(f & 63u), m0 = small_int_f((f >> 6) & 63u);
    const float sc1 = small_int_f((f >> 12) & 63u), m1 = small_int_f((f >> 18) & 63u);
    return d * (sc0 * acc_lo + sc1 * acc_hi) -
           dmin * (m0 * s.sum[c] + m1 * s.sum[kChunks + c]);
  } else {
    const unsigned p = (c % 8) % 4, sh_lo = 2 * (p / 2), sh_hi = sh_lo + 4;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint32_t q = word(w.lo, v), h = word(w.aux, v);
      const float4 xl = s.xv[v * kChunks + c], xh = s.xv[(4 + v) * kChunks + c];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t ql = (q >> (8 * e)) & 0xFFu, qh = (h >> (8 * e)) & 0xFFu;
        const uint32_t q_lo = (ql & 15u) | ((qh >> sh_lo) & 3u) << 4;
        const uint32_t q_hi = (ql >> 4) | ((qh >> sh_hi) & 3u) << 4;
        const float x_lo = e == 0 ? xl.x : e == 1 ? xl.y : e == 2 ? xl.z : xl.w;
        const float x_hi = e == 0 ? xh.x : e == 1 ? xh.y : e == 2 ? xh.z : xh.w;
        acc_lo += q6_f(q_lo) * x_lo;
        acc_hi += q6_f(q_hi) * x_hi;
      }
    }
    const float d = f16_bits(w.sd >> 16);
    const float s_lo = static_cast<float>(static_cast<int8_t>(w.sd & 0xFFu));
    const float s_hi = static_cast<float>(static_cast<int8_t>((w.sd >> 8) & 0xFFu));
    return d * (s_lo * acc_lo + s_hi * acc_hi);
  }
}

// This lane's share of one row's dot product (chunks lane, lane + 32, ...); the caller reduces
// over the warp.
template <Fmt F, unsigned K>
__device__ __forceinline__ float row_partial(const uint8_t* row, const StagedX<K>& s) {
  constexpr unsigned kChunks = K / 32;
  constexpr unsigned kPerLane = (kChunks + kWave - 1) / kWave;
  const unsigned lane = threadIdx.x % kWave;
  ChunkW cw[kPerLane];
#pragma unroll
  for (unsigned u = 0; u < kPerLane; ++u)
    if (lane + u * kWave < kChunks)
      cw[u] = load_chunk<F>(row, K, lane + u * kWave);
  float acc = 0.0f;
#pragma unroll
  for (unsigned u = 0; u < kPerLane; ++u)
    if (lane + u * kWave < kChunks)
      acc += chunk_dot<F, K>(cw[u], s, lane + u * kWave);
  return acc;
}

// y[r] = W[r] . x for rows [first, first + count): the grid's warps (warp_id of warp_count) stride
// over groups of kRows rows; each lane loads all its chunks of the kRows rows before it computes.
// Lane 0 stores.
template <Fmt F, unsigned K, int kRows>
__device__ inline void rows_dot(const uint8_t* w, float* y, unsigned first, unsigned count,
                                const StagedX<K>& s, unsigned warp_id, unsigned warp_count) {
  constexpr unsigned kChunks = K / 32;
  constexpr unsigned kPerLane = (kChunks + kWave - 1) / kWave;
  constexpr std::size_t kRowBytes = row_bytes<F>(K);
  const unsigned lane = threadIdx.x % kWave, end = first + count;
  for (unsigned r0 = first + warp_id * kRows; r0 < end; r0 += warp_count * kRows) {
    ChunkW cw[kRows][kPerLane];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (unsigned u = 0; u < kPerLane; ++u) {
        const unsigned c = lane + u * kWave;
        if (r0 + r < end && c < kChunks)
          cw[r][u] = load_chunk<F>(w + (r0 + r) * kRowBytes, K, c);
      }
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      float acc = 0.0f;
#pragma unroll
      for (unsigned u = 0; u < kPerLane; ++u) {
        const unsigned c = lane + u * kWave;
        if (r0 + r < end && c < kChunks)
          acc += chunk_dot<F, K>(cw[r][u], s, c);
      }
      acc = wave_sum(acc);
      if (lane == 0 && r0 + r < end)
        y[r0 + r] = acc;
    }
  }
}

}  // namespace gemv

}  // namespace miso::kernels
