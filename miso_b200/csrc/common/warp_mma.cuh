#pragma once

// Warp-level tensor-core fragments (sm_80+ mma.sync m16n8k16, ldmatrix, movmatrix) and the fp16
// hi / lo split, as inline functions only (no device variables), so that the drop-in kernel
// headers, which the reference engine compiles into several of its own translation units, can
// include them.

#include <cuda_fp16.h>

#include <cstdint>

namespace miso::dev {

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

// Transpose of an 8x8 b16 matrix held in the standard fragment layout (lane i: row i/4,
// columns 2(i%4), 2(i%4)+1).
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// D = A(16x16, row) * B(16x8, col) + D, f16 inputs, f32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo_elem, float hi_elem) {
  const __half2 h = __floats2half2_rn(lo_elem, hi_elem);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Two-term fp16 split of an fp32 pair: hi = fp16(x), lo = fp16(x - hi). hi + lo carries ~22
// significant bits, so products against exact fp16 operands keep fp32-level accuracy.
__device__ __forceinline__ void split_half2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const __half l0 = __float2half_rn(x0 - __half2float(h0));
  const __half l1 = __float2half_rn(x1 - __half2float(h1));
  const __half2 H = __halves2half2(h0, h1), L = __halves2half2(l0, l1);
  hi = *reinterpret_cast<const uint32_t*>(&H);
  lo = *reinterpret_cast<const uint32_t*>(&L);
}

// Byte permute of two 32-bit words (PTX prmt.b32).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// L2 policy for data read once (evict first).
__device__ __forceinline__ uint64_t stream_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 16-byte read-only global load of streamed data: no L1 allocation, L2 evict-first.
__device__ __forceinline__ uint4 ld_stream16(const void* ptr, uint64_t policy) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr), "l"(policy));
  return v;
}

}  // namespace miso::dev
