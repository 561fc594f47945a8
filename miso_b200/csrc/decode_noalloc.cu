// miso_attn_decode_noalloc: the batched split-K decode without caller-provided scratch.
//
// Who needs it: callers that cannot allocate device memory for the decode's scratch. Examples are
// a serving framework that reserves nearly all of the GPU's memory up front for its own pool and
// allows no allocation outside it, a plugin loaded into such a host that only receives the
// tensors it works on, and a latency-critical decode loop that cannot afford cudaMalloc's
// implicit device-wide synchronisation. They pass only inputs and outputs; the scratch (per-
// segment arrival counters and per-CTA partial results) lives in the library itself, in the
// file-scope __device__ array below, which the CUDA module loader places on every GPU that loads
// the library and keeps there until the process exits.
//
// Fixed limits (checked, MISO_ERR_LIMIT beyond them): batch <= 256 sequences and at most 160
// CTAs (the B200 has 148 SMs, one CTA each). The array is 2,643,968 bytes per GPU.
//
// The array is shared by every call on a device and keeps the last call's contents. Each call
// zeroes the counters it uses (an async memset on its own stream) before its kernel, so leftovers
// of an earlier call, even an aborted one, do not leak in; but two calls that overlap on the GPU
// (different streams with no ordering between them) use the same memory and race.
//
// Host code cannot use the array's name as a device address (there it names a host-side stand-in).
// The first call on each device, with that device current, looks the address up with
// cudaGetSymbolAddress and remembers it; make that first call before any stream capture. A
// lookup that fails is not remembered: that call returns the error and the next call retries.
//
// This file is part of the single translation unit of capi.cu (included at its end), next to the
// kernel and the helpers it reuses.

namespace {

constexpr unsigned kNoAllocMaxBatch = 256;
constexpr unsigned kNoAllocMaxCtas = 160;
constexpr size_t kNoAllocCounterBytes = (2 * kNoAllocMaxBatch * sizeof(int) + 255) & ~size_t(255);
constexpr size_t kNoAllocBytes =
    kNoAllocCounterBytes + size_t(2) * kNoAllocMaxCtas * miso::fast::decode::kPartFloats * sizeof(float);
static_assert(kNoAllocBytes == 2643968, "size stated in the comment above and in the docs");

}  // namespace

static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[kNoAllocBytes];

namespace {

// Device address of g_decode_noalloc_scratch on each device; null until a lookup succeeded.
void* g_noalloc_scratch[kMaxDevices] = {};
std::mutex g_noalloc_mutex;

// Device address of the scratch array on the current device. Only a successful lookup is kept:
// a failed one (for example, a first call made during stream capture) returns its error and the
// next call looks again.
int noalloc_scratch(void** out) {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices)
    return MISO_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t r = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (r != cudaSuccess)
      return static_cast<int>(r);
    if (p == nullptr)
      return MISO_ERR_NO_DEVICE;
    g_noalloc_scratch[dev] = p;
  }
  *out = g_noalloc_scratch[dev];
  return MISO_OK;
}

}  // namespace

extern "C" int miso_attn_decode_noalloc(const miso_attn_decode_params* p, void* stream) {
  namespace dec = miso::fast::decode;
  if (p == nullptr || p->q == nullptr || p->qg == nullptr || p->k_pool == nullptr ||
      p->v_pool == nullptr || p->kv_row == nullptr || p->lens == nullptr || p->core == nullptr ||
      p->batch == 0 || p->pool_rows == 0 || p->pool_rows >= (uint64_t(1) << 31) ||
      !aligned16(p->k_pool) || !aligned16(p->v_pool) ||
      (reinterpret_cast<uintptr_t>(p->q) & 7u) != 0)
    return MISO_ERR_INVALID;
  if (p->batch > kNoAllocMaxBatch)
    return MISO_ERR_LIMIT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != MISO_OK)
    return st;
  if ((st = tensor_map_encoder()) != MISO_OK)
    return st;
  void* scratch = nullptr;
  if ((st = noalloc_scratch(&scratch)) != MISO_OK)
    return st;
  const unsigned ctas = d->sms < int(kNoAllocMaxCtas) ? unsigned(d->sms) : kNoAllocMaxCtas;
  CUtensorMap kmap, vmap;
  if ((st = kv_pool_map(&kmap, p->k_pool, p->pool_rows)) != MISO_OK ||
      (st = kv_pool_map(&vmap, p->v_pool, p->pool_rows)) != MISO_OK)
    return st;
  cudaError_t e = cudaMemsetAsync(scratch, 0, size_t(2) * p->batch * sizeof(int),
                                  as_stream(stream));
  if (e != cudaSuccess)
    return static_cast<int>(e);
  dec::Args a;
  a.q = p->q;
  a.qg = p->qg;
  a.kv_row = p->kv_row;
  a.lens = p->lens;
  a.core = p->core;
  a.counters = static_cast<int*>(scratch);
  a.parts = reinterpret_cast<float*>(static_cast<char*>(scratch) + kNoAllocCounterBytes);
  a.batch = p->batch;
  a.qg_stride = p->qg_stride;
  dec::decode_kernel<<<ctas, dec::kThreads, dec::kSmemBytes, as_stream(stream)>>>(kmap, vmap, a);
  return launch_status();
}
