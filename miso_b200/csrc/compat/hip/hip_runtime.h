#pragma once

// Source-compatibility shim: lets HIP host sources of the reference engine and tests
// (src/engine/*.hip, tests/*.hip) compile as CUDA unchanged. Maps the HIP runtime names those
// files use onto the CUDA runtime; the kernels themselves come from the drop-in headers.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

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

#define hipMalloc cudaMalloc
#define hipFree cudaFree
#define hipMemcpy cudaMemcpy
#define hipMemcpyAsync cudaMemcpyAsync
#define hipMemset cudaMemset
#define hipMemsetAsync cudaMemsetAsync
#define hipHostMalloc(ptr, size, flags) cudaHostAlloc((ptr), (size), (flags))
#define hipHostFree cudaFreeHost
#define hipGetLastError cudaGetLastError
#define hipPeekAtLastError cudaPeekAtLastError
#define hipDeviceSynchronize cudaDeviceSynchronize
#define hipStreamCreate cudaStreamCreate
#define hipStreamDestroy cudaStreamDestroy
#define hipStreamSynchronize cudaStreamSynchronize
#define hipEventCreate cudaEventCreate
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
