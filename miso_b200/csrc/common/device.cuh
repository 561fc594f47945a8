#pragma once

// sm_100a device building blocks shared by the fast kernels: shared-memory addressing, mbarriers
// with bounded waits, TMA tile loads (the warp-level MMA fragments are in warp_mma.cuh).
//
// Every wait on an mbarrier is bounded (SM clock cycles). When a wait gives up, the kernel records
// MISO_STATUS_TIMEOUT and the waiting site in the library's device status word and stops issuing
// work instead of spinning forever; the host reads the word with miso_device_status().

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "warp_mma.cuh"

namespace miso::dev {

// Device status word codes (also in include/miso_cuda.h as MISO_STATUS_*).
constexpr int kStatusOk = 0;
constexpr int kStatusTimeout = 1;

// Bound on any single mbarrier wait, in SM clock cycles (the per-SM cycle counter is monotonic):
// 4e9 cycles, about 2 s at the B200's 1.9-2.0 GHz. Legitimate waits here are microseconds.
constexpr long long kWaitLimitCycles = 4000000000ll;

// Device status word of this library (one per device per loaded copy of the library).
__device__ int g_status = 0;

// Records the first failure of the process on this device: low byte = code, bits 8.. = the site
// (which kernel and which wait) that hit it.
__device__ __forceinline__ void set_status(int code, int site = 0) {
  atomicCAS(&g_status, kStatusOk, code | (site << 8));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes initialised barriers visible to the async proxy (TMA) before first use.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          bar),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and records a timeout and
// `site` in the status word) if it has not completed within kWaitLimitCycles.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int site = 0) {
  if (mbar_try_wait(bar, parity))
    return true;
  const long long t0 = clock64();
  for (unsigned i = 1;; ++i) {
    if (mbar_try_wait(bar, parity))
      return true;
    if ((i & 255u) == 0 && clock64() - t0 > kWaitLimitCycles) {
      set_status(kStatusTimeout, site);
      return false;
    }
  }
}

// Non-blocking test of the phase with the given parity.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA) writes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMA --------------------------------------------------------------------------------------

// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global to
// shared memory, completion signalled on `bar` (complete_tx).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of one box into shared memory; completion is signalled on `bar` (complete_tx).
// x is the innermost coordinate in elements; x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Same with an L2 eviction-priority policy (e.g. evict-first for data streamed exactly once).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// Bulk prefetch of `bytes` (a multiple of 16) at the 16-byte aligned global address `p` into L2.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a box written by TMA with
// CU_TENSOR_MAP_SWIZZLE_128B and 128-byte rows (box base aligned to 1024 bytes).
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + (((chunk ^ row) & 7u) << 4);
}

__device__ __forceinline__ void named_bar_sync(unsigned id, unsigned threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace miso::dev
