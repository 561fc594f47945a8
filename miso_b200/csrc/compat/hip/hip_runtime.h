#pragma once

// Source-compatibility shim: lets HIP host sources of the reference engine and tests
// (src/engine/*.hip, tests/*.hip) compile as CUDA unchanged. Maps the HIP runtime names those
// files use onto the CUDA runtime; the kernels themselves come from the drop-in headers.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>

// The reference spells binary16 `_Float16`. nvcc 12.9's device front end stops with "unsupported
// float variant" on C++20 library code instantiated for _Float16 even where only host code uses it
// (std::vector<_Float16>::resize), so after this header the name means CUDA's __half: the same
// 2-byte IEEE binary16 layout, with round-to-nearest-even conversions from and to float on the
// host and the device. (<algorithm> is included because HIP's runtime header provides it.)
#define _Float16 __half

typedef cudaStream_t hipStream_t;
typedef cudaError_t hipError_t;
typedef cudaEvent_t hipEvent_t;
typedef cudaMemcpyKind hipMemcpyKind;
typedef cudaGraph_t hipGraph_t;
typedef cudaGraphExec_t hipGraphExec_t;

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
#define hipSetDevice cudaSetDevice
#define hipGetDevice cudaGetDevice
#define hipRuntimeGetVersion cudaRuntimeGetVersion
#define hipStreamBeginCapture cudaStreamBeginCapture
#define hipStreamEndCapture cudaStreamEndCapture
#define hipStreamCaptureModeGlobal cudaStreamCaptureModeGlobal
#define hipGraphLaunch cudaGraphLaunch
#define hipGraphDestroy cudaGraphDestroy
#define hipGraphExecDestroy cudaGraphExecDestroy

// Pinned host allocation; HIP's flags argument defaults to 0 and its default / portable / mapped
// bits have the CUDA values.
inline cudaError_t hipHostMalloc(void** ptr, size_t size, unsigned int flags = 0) {
  return cudaHostAlloc(ptr, size, flags);
}
template <class T>
inline cudaError_t hipHostMalloc(T** ptr, size_t size, unsigned int flags = 0) {
  return cudaHostAlloc(reinterpret_cast<void**>(ptr), size, flags);
}

// Device properties: CUDA's, plus HIP's architecture-name field (here "sm_<major><minor>").
struct hipDeviceProp_t : cudaDeviceProp {
  char gcnArchName[256];
};
inline cudaError_t hipGetDeviceProperties(hipDeviceProp_t* p, int device) {
  const cudaError_t e = cudaGetDeviceProperties(static_cast<cudaDeviceProp*>(p), device);
  if (e == cudaSuccess)
    std::snprintf(p->gcnArchName, sizeof p->gcnArchName, "sm_%d%d", p->major, p->minor);
  return e;
}

// HIP keeps the older five-argument form (error node and log buffer, unused here).
inline cudaError_t hipGraphInstantiate(hipGraphExec_t* exec, hipGraph_t graph, void* error_node,
                                       char* log, size_t log_size) {
  (void)error_node, (void)log, (void)log_size;
  return cudaGraphInstantiate(exec, graph, 0);
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
