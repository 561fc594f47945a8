#pragma once

// Source-compatibility shim: lets HIP host sources of the reference engine and tests
// (src/engine/*.hip, tests/*.hip) compile as CUDA unchanged. Maps the HIP runtime names those
// files use onto the CUDA runtime; the kernels themselves come from the drop-in headers.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

// The reference spells binary16 `_Float16`. nvcc 12.9's device front end stops with "unsupported
// float variant" on C++20 library code instantiated for _Float16 even where only host code uses it
// (std::vector<_Float16>::resize), so after this header the name means CUDA's __half: the same
// 2-byte IEEE binary16 layout, with round-to-nearest-even conversions from and to float on the
// host and the device. (<algorithm> is included because HIP's runtime header provides it.)
#define _Float16 __half

typedef cudaStream_t hipStream_t;
typedef cudaError_t hipError_t;
typedef cudaEvent_t hipEvent_t;
typedef cudaDeviceProp hipDeviceProp_t;
typedef cudaMemcpyKind hipMemcpyKind;

#define hipSuccess cudaSuccess
#define hipErrorInvalidValue cudaErrorInvalidValue
#define hipMemcpyHostToDevice cudaMemcpyHostToDevice
#define hipMemcpyDeviceToHost cudaMemcpyDeviceToHost
#define hipMemcpyDeviceToDevice cudaMemcpyDeviceToDevice
#define hipMemcpyHostToHost cudaMemcpyHostToHost
#define hipMemcpyDefault cudaMemcpyDefault
#define hipHostMallocDefault cudaHostAllocDefault
#define hipStreamDefault cudaStreamDefault
#define hipStreamNonBlocking cudaStreamNonBlocking
#define hipEventDefault cudaEventDefault
#define hipEventDisableTiming cudaEventDisableTiming

#define hipMalloc cudaMalloc
#define hipFree cudaFree
#define hipMemcpy cudaMemcpy
#define hipMemcpyAsync cudaMemcpyAsync
#define hipMemset cudaMemset
#define hipMemsetAsync cudaMemsetAsync
#define hipHostFree cudaFreeHost
#define hipGetLastError cudaGetLastError
#define hipPeekAtLastError cudaPeekAtLastError
#define hipDeviceSynchronize cudaDeviceSynchronize
#define hipStreamCreate cudaStreamCreate
#define hipStreamCreateWithFlags cudaStreamCreateWithFlags
#define hipStreamDestroy cudaStreamDestroy
#define hipStreamSynchronize cudaStreamSynchronize
#define hipEventCreate cudaEventCreate
#define hipEventCreateWithFlags cudaEventCreateWithFlags
#define hipEventDestroy cudaEventDestroy
#define hipEventRecord cudaEventRecord
#define hipEventSynchronize cudaEventSynchronize
#define hipEventElapsedTime cudaEventElapsedTime
#define hipGetErrorName cudaGetErrorName
#define hipGetErrorString cudaGetErrorString
#define hipGetDeviceCount cudaGetDeviceCount
#define hipGetDeviceProperties cudaGetDeviceProperties
#define hipSetDevice cudaSetDevice
#define hipGetDevice cudaGetDevice

// Pinned host allocation; HIP's flags argument defaults to 0 and its default / portable / mapped
// bits have the CUDA values.
inline cudaError_t hipHostMalloc(void** ptr, size_t size, unsigned int flags = 0) {
  return cudaHostAlloc(ptr, size, flags);
}
template <class T>
inline cudaError_t hipHostMalloc(T** ptr, size_t size, unsigned int flags = 0) {
  return cudaHostAlloc(reinterpret_cast<void**>(ptr), size, flags);
}

// HIP's width-taking shuffles over the full warp.
#if defined(__CUDACC__)
template <class T>
__device__ __forceinline__ T __shfl_xor(T v, int mask, int width = warpSize) {
  return __shfl_xor_sync(0xffffffffu, v, mask, width);
}
template <class T>
__device__ __forceinline__ T __shfl(T v, int src, int width = warpSize) {
  return __shfl_sync(0xffffffffu, v, src, width);
}
#endif
