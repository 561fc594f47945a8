#pragma once

// CUDA counterpart of the reference's src/hip_util.hpp (:1-57): error check that throws, an
// owning device buffer, and the MISO_HIP_CHECK macro, with the same names and behaviour so the
// reference engine and tests compile unchanged against CUDA.

#include <cuda_runtime.h>

#include <cstddef>
#include <stdexcept>
#include <string>
#include <vector>

namespace miso {

inline void hip_check(cudaError_t err, const char* expr) {
  if (err != cudaSuccess) {
    throw std::runtime_error(std::string(expr) + " failed: " + cudaGetErrorName(err) + " (" +
                             cudaGetErrorString(err) + ")");
  }
}

// CUDA-named alias of hip_check.
inline void cuda_check(cudaError_t err, const char* expr) { hip_check(err, expr); }

// Owning device allocation of `size()` elements of T. Move-only.
template <class T>
class DeviceBuffer {
 public:
  explicit DeviceBuffer(std::size_t n) : n_(n) {
    hip_check(cudaMalloc(reinterpret_cast<void**>(&p_), n * sizeof(T)), "cudaMalloc");
  }
  explicit DeviceBuffer(const std::vector<T>& host) : DeviceBuffer(host.size()) {
    hip_check(cudaMemcpy(p_, host.data(), n_ * sizeof(T), cudaMemcpyHostToDevice),
              "cudaMemcpy H2D");
  }
  DeviceBuffer(DeviceBuffer&& o) noexcept : p_(o.p_), n_(o.n_) {
    o.p_ = nullptr;
    o.n_ = 0;
  }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(DeviceBuffer&&) = delete;
  ~DeviceBuffer() {
    if (p_ != nullptr)
      (void)cudaFree(p_);
  }

  T* data() const { return p_; }
  std::size_t size() const { return n_; }

  std::vector<T> to_host() const {
    std::vector<T> host(n_);
    hip_check(cudaMemcpy(host.data(), p_, n_ * sizeof(T), cudaMemcpyDeviceToHost),
              "cudaMemcpy D2H");
    return host;
  }

 private:
  T* p_ = nullptr;
  std::size_t n_;
};

}  // namespace miso

#define MISO_HIP_CHECK(expr) ::miso::hip_check((expr), #expr)
#define MISO_CUDA_CHECK(expr) ::miso::hip_check((expr), #expr)
