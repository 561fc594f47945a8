#pragma once

// Addresses of binary16 arrays in kernel parameter structs. The reference's parameter structs
// type these fields _Float16* (e.g. kernels/qgemm.hpp:24-37, moe_prefill.hpp:223-235), and its
// engine passes _Float16 buffers. nvcc accepts _Float16 in host code but not in device code, so
// the fields hold __half pointers (the same 2-byte IEEE binary16 layout) and convert implicitly,
// on the host, from _Float16 pointers. Under the HIP compatibility header _Float16 already names
// __half, and the extra constructors are left out.

#include <cuda_fp16.h>

namespace miso::kernels {

struct F16In {
  const __half* p;
  __host__ __device__ F16In(const __half* q = nullptr) : p(q) {}
#ifndef _Float16
  F16In(const _Float16* q) : p(reinterpret_cast<const __half*>(q)) {}
#endif
};

struct F16Out {
  __half* p;
  __host__ __device__ F16Out(__half* q = nullptr) : p(q) {}
#ifndef _Float16
  F16Out(_Float16* q) : p(reinterpret_cast<__half*>(q)) {}
#endif
};

}  // namespace miso::kernels
