// C entry points over the reference's own weight-format code (src/dequant.cpp, src/repack.cpp,
// compiled from the reference's sources where they lie into oracle/_ref/) — TEST INFRASTRUCTURE
// ONLY: tests/test_oracle_quant.py pins the numpy restatement (oracle/quant.py) against it.
// Every function returns 0, or -1 when the reference code throws.

#include <cstddef>
#include <cstdint>
#include <span>

#include "dequant.hpp"
#include "repack.hpp"

namespace {

std::span<const std::byte> in(const void* p, std::size_t n) {
  return {static_cast<const std::byte*>(p), n};
}
std::span<std::byte> out(void* p, std::size_t n) { return {static_cast<std::byte*>(p), n}; }

}  // namespace

extern "C" {

int ref_dequant(int type, const void* src, std::size_t src_bytes, float* dst, std::size_t n) {
  try {
    miso::dequantize(static_cast<miso::gguf::GgmlType>(type), in(src, src_bytes), {dst, n});
    return 0;
  } catch (...) {
    return -1;
  }
}

int ref_repack_q4k(const void* src, std::size_t bytes, void* dst) {
  try {
    miso::repack_q4k(in(src, bytes), out(dst, bytes));
    return 0;
  } catch (...) {
    return -1;
  }
}

int ref_repack_q6k(const void* src, std::size_t bytes, std::size_t row_elements, void* dst,
                   std::size_t dst_bytes) {
  try {
    miso::repack_q6k(in(src, bytes), row_elements, out(dst, dst_bytes));
    return 0;
  } catch (...) {
    return -1;
  }
}

std::size_t ref_q6k_r1_row_bytes(std::size_t row_elements) {
  return miso::q6k_r1_row_bytes(row_elements);
}

}  // extern "C"
