// C ABI of the B200 attention hot path (declared in include/miso_cuda.h).
//
// Drop-in entry points launch the reference-named kernels of kernels/*.hpp with the geometry the
// reference engine uses; fast entry points launch the sm_100a kernels of fast/*.cuh with
// library-chosen geometry. Nothing here throws: every entry point returns MISO_OK, a negative
// MISO_ERR_* for a rejected argument, or the positive cudaError_t of the launch.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include "miso_cuda.h"

#include "common/device.cuh"
#include "fast/attn_decode.cuh"
#include "fast/attn_prefill_tc.cuh"
#include "fast/attn_prep.cuh"
#include "fast/deltanet_step_batched.cuh"
#include "fast/deltanet_prefill_tc.cuh"
#include "kernels/attention_decode.hpp"
#include "kernels/attention_prefill.hpp"
#include "kernels/deltanet_chunk.hpp"
#include "kernels/deltanet_step.hpp"

namespace k = miso::kernels;

// ---- the C structs are the reference Params, field for field ---------------------------------

#define MISO_SAME_LAYOUT(C, CPP, field) \
  static_assert(offsetof(C, field) == offsetof(CPP, field), #C "." #field)

static_assert(sizeof(miso_attn_prep_params) == sizeof(k::AttnPrepParams), "AttnPrepParams size");
MISO_SAME_LAYOUT(miso_attn_prep_params, k::AttnPrepParams, k_cache);
MISO_SAME_LAYOUT(miso_attn_prep_params, k::AttnPrepParams, q);
MISO_SAME_LAYOUT(miso_attn_prep_params, k::AttnPrepParams, pos);
MISO_SAME_LAYOUT(miso_attn_prep_params, k::AttnPrepParams, eps);
static_assert(sizeof(miso_attn_prep_batch_params) == sizeof(k::AttnPrepBatchParams), "batch");
MISO_SAME_LAYOUT(miso_attn_prep_batch_params, k::AttnPrepBatchParams, n);
MISO_SAME_LAYOUT(miso_attn_prep_batch_params, k::AttnPrepBatchParams, proj_stride);
static_assert(sizeof(miso_attn_split_params) == sizeof(k::AttnSplitParams), "AttnSplitParams");
MISO_SAME_LAYOUT(miso_attn_split_params, k::AttnSplitParams, part_o);
MISO_SAME_LAYOUT(miso_attn_split_params, k::AttnSplitParams, n_splits);
static_assert(sizeof(miso_attn_combine_params) == sizeof(k::AttnCombineParams), "combine");
MISO_SAME_LAYOUT(miso_attn_combine_params, k::AttnCombineParams, core);
MISO_SAME_LAYOUT(miso_attn_combine_params, k::AttnCombineParams, n_splits);
static_assert(sizeof(miso_attn_prefill_params) == sizeof(k::AttnPrefillParams), "prefill");
MISO_SAME_LAYOUT(miso_attn_prefill_params, k::AttnPrefillParams, core);
MISO_SAME_LAYOUT(miso_attn_prefill_params, k::AttnPrefillParams, qg_stride);
static_assert(sizeof(miso_deltanet_step_params) == sizeof(k::DeltaNetStepParams), "step");
MISO_SAME_LAYOUT(miso_deltanet_step_params, k::DeltaNetStepParams, state);
MISO_SAME_LAYOUT(miso_deltanet_step_params, k::DeltaNetStepParams, eps);
static_assert(sizeof(miso_deltanet_seq_params) == sizeof(k::DeltaNetSeqParams), "seq");
MISO_SAME_LAYOUT(miso_deltanet_seq_params, k::DeltaNetSeqParams, n);
MISO_SAME_LAYOUT(miso_deltanet_seq_params, k::DeltaNetSeqParams, qkv_stride);
static_assert(sizeof(miso_deltanet_conv_params) == sizeof(k::DeltaNetConvParams), "conv");
MISO_SAME_LAYOUT(miso_deltanet_conv_params, k::DeltaNetConvParams, log_a);
MISO_SAME_LAYOUT(miso_deltanet_conv_params, k::DeltaNetConvParams, n);
static_assert(sizeof(miso_deltanet_chunk_params) == sizeof(k::DeltaNetChunkParams), "chunk");
MISO_SAME_LAYOUT(miso_deltanet_chunk_params, k::DeltaNetChunkParams, sq);
MISO_SAME_LAYOUT(miso_deltanet_chunk_params, k::DeltaNetChunkParams, eps);

namespace {

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MISO_OK : static_cast<int>(e);
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- per-device state ----------------------------------------------------------------------

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::once_flag once;
  int status = MISO_OK;
  int sms = 0;
};

DeviceInfo g_dev[kMaxDevices];

// Streams and events of the pipelined DeltaNet prefill (one set per device, created on first use):
// the per-piece front launches, chain launches and gate launches run on three streams that fork
// from and join back into the caller's stream. The mutex keeps one call's enqueue sequence whole
// (the events are reused from call to call).
constexpr int kDnMaxPieces = 64;
constexpr unsigned kDnPieceChunks = 32;  // chunks of 64 tokens per piece (8, 16, 64 measured slower)
constexpr unsigned kDnFirstPieceChunks = 16;  // the first piece
struct DnPipe {
  std::once_flag once;
  int status = MISO_OK;
  std::mutex mu;
  cudaStream_t front = nullptr, chain = nullptr, gate = nullptr;
  cudaEvent_t fork = nullptr, front_done[kDnMaxPieces] = {}, chain_done[kDnMaxPieces] = {};
  cudaEvent_t join_front = nullptr, join_gate = nullptr;
};
DnPipe g_dn_pipe[kMaxDevices];

int dn_pipe(DnPipe** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices)
    return MISO_ERR_NO_DEVICE;
  DnPipe& q = g_dn_pipe[dev];
  std::call_once(q.once, [&] {
    int lo = 0, hi = 0;
    cudaError_t r = cudaDeviceGetStreamPriorityRange(&lo, &hi);
    // The chain (the critical path) at the highest priority, so that its CTAs are placed before
    // waiting front and gate CTAs whenever an SM frees up.
    if (r == cudaSuccess)
      r = cudaStreamCreateWithPriority(&q.chain, cudaStreamNonBlocking, hi);
    if (r == cudaSuccess)
      r = cudaStreamCreateWithPriority(&q.front, cudaStreamNonBlocking, lo);
    if (r == cudaSuccess)
      r = cudaStreamCreateWithPriority(&q.gate, cudaStreamNonBlocking, lo);
    const unsigned fl = cudaEventDisableTiming;
    if (r == cudaSuccess)
      r = cudaEventCreateWithFlags(&q.fork, fl);
    if (r == cudaSuccess)
      r = cudaEventCreateWithFlags(&q.join_front, fl);
    if (r == cudaSuccess)
      r = cudaEventCreateWithFlags(&q.join_gate, fl);
    for (int i = 0; r == cudaSuccess && i < kDnMaxPieces; ++i) {
      r = cudaEventCreateWithFlags(&q.front_done[i], fl);
      if (r == cudaSuccess)
        r = cudaEventCreateWithFlags(&q.chain_done[i], fl);
    }
    q.status = r == cudaSuccess ? MISO_OK : static_cast<int>(r);
  });
  if (q.status != MISO_OK)
    return q.status;
  *out = &q;
  return MISO_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices)
    return MISO_ERR_NO_DEVICE;
  DeviceInfo& d = g_dev[dev];
  std::call_once(d.once, [&] {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      d.status = MISO_ERR_NO_DEVICE;
      return;
    }
    if (major != 10) {
      d.status = MISO_ERR_NO_DEVICE;
      return;
    }
    d.sms = sms;
    cudaError_t a = cudaFuncSetAttribute(miso::fast::decode::decode_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(miso::fast::decode::kSmemBytes));
    if (a == cudaSuccess)
      a = cudaFuncSetAttribute(miso::fast::prefill::prefill_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(miso::fast::prefill::kSmemBytes));
    if (a == cudaSuccess)
      a = cudaFuncSetAttribute(miso::fast::dnstep::step_batched_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(miso::fast::dnstep::kSmemBytes));
    if (a == cudaSuccess)
      a = cudaFuncSetAttribute(miso::fast::dnpf::front_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(miso::fast::dnpf::kFrontSmemBytes));
    if (a == cudaSuccess)
      a = cudaFuncSetAttribute(miso::fast::dnpf::chain_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(miso::fast::dnpf::kChainSmemBytes));
    d.status = a == cudaSuccess ? MISO_OK : static_cast<int>(a);
  });
  *out = &d;
  return d.status;
}

int tensor_map_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr ? MISO_OK : MISO_ERR_DRIVER;
}

// 2-D fp16 map over a [rows][256] pool; box = 64 dims x 64 rows, 128-byte swizzle.
int kv_pool_map(CUtensorMap* map, const void* pool, uint64_t rows) {
  const cuuint64_t dims[2] = {256, rows};
  const cuuint64_t strides[1] = {256 * sizeof(uint16_t)};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(pool),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MISO_OK : MISO_ERR_INVALID;
}

// fp16 tensor map with a 128-byte swizzle; dims / box innermost first, strides in bytes for
// dims 1..rank-1.
int f16_map(CUtensorMap* map, const void* ptr, cuuint32_t rank, const cuuint64_t* dims,
            const cuuint64_t* strides, const cuuint32_t* box) {
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(ptr),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MISO_OK : MISO_ERR_INVALID;
}

// 2-D fp32 tensor map, by default without swizzle; dims / box innermost first, row stride in
// bytes.
int f32_map(CUtensorMap* map, const void* ptr, const cuuint64_t* dims, const cuuint64_t* strides,
            const cuuint32_t* box, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MISO_OK : MISO_ERR_INVALID;
}

size_t decode_counter_bytes(unsigned batch) {
  return (size_t(2) * batch * sizeof(int) + 255) & ~size_t(255);
}

}  // namespace

extern "C" {

const char* miso_version(void) { return "miso_b200 0.1 (sm_100a)"; }

unsigned miso_attn_n_splits(unsigned len, unsigned max_splits) {
  return k::attn_n_splits(len, max_splits);
}

unsigned miso_attn_prefill_items(unsigned n) { return k::attn_prefill_items(n); }

int miso_device_status(int reset, int* status) {
  if (status == nullptr)
    return MISO_ERR_INVALID;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess)
    return static_cast<int>(e);
  e = cudaMemcpyFromSymbol(status, miso::dev::g_status, sizeof(int));
  if (e != cudaSuccess)
    return static_cast<int>(e);
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(miso::dev::g_status, &zero, sizeof(int));
    if (e != cudaSuccess)
      return static_cast<int>(e);
  }
  return MISO_OK;
}

// ---- drop-in family ---------------------------------------------------------------------------

int miso_attn_prep(const miso_attn_prep_params* p, void* stream) {
  if (p == nullptr || p->qg == nullptr || p->k == nullptr || p->v == nullptr ||
      p->q_norm == nullptr || p->k_norm == nullptr || p->inv_freq == nullptr ||
      p->k_cache == nullptr || p->v_cache == nullptr || p->q == nullptr || p->pos >= p->max_ctx ||
      !aligned16(p->qg) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->q_norm) ||
      !aligned16(p->k_norm) || !aligned16(p->q) || !aligned16(p->k_cache) ||
      !aligned16(p->v_cache))
    return MISO_ERR_INVALID;
  k::attn_prep_kernel<256><<<18, 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::AttnPrepParams*>(p));
  return launch_status();
}

int miso_attn_prep_batch(const miso_attn_prep_batch_params* p, void* stream) {
  if (p == nullptr || p->tok0.qg == nullptr || p->tok0.k == nullptr || p->tok0.v == nullptr ||
      p->tok0.q_norm == nullptr || p->tok0.k_norm == nullptr || p->tok0.inv_freq == nullptr ||
      p->tok0.k_cache == nullptr || p->tok0.v_cache == nullptr || p->tok0.q == nullptr ||
      uint64_t(p->tok0.pos) + p->n > p->tok0.max_ctx || p->proj_stride % 4 != 0 ||
      !aligned16(p->tok0.qg) || !aligned16(p->tok0.k) || !aligned16(p->tok0.v) ||
      !aligned16(p->tok0.q_norm) || !aligned16(p->tok0.k_norm) || !aligned16(p->tok0.q) ||
      !aligned16(p->tok0.k_cache) || !aligned16(p->tok0.v_cache))
    return MISO_ERR_INVALID;
  if (p->n == 0)
    return MISO_OK;
  k::attn_prep_batch_kernel<256><<<p->n * 18, 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::AttnPrepBatchParams*>(p));
  return launch_status();
}

int miso_attn_split(const miso_attn_split_params* p, void* stream) {
  if (p == nullptr || p->q == nullptr || p->k_cache == nullptr || p->v_cache == nullptr ||
      p->part_m == nullptr || p->part_l == nullptr || p->part_o == nullptr || p->n_splits == 0 ||
      p->len == 0 || p->len > p->max_ctx || p->n_splits > 65535 || !aligned16(p->q) ||
      !aligned16(p->k_cache) ||
      !aligned16(p->v_cache) || !aligned16(p->part_o))
    return MISO_ERR_INVALID;
  k::attn_split_kernel<256><<<dim3(p->n_splits, 2), 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::AttnSplitParams*>(p));
  return launch_status();
}

int miso_attn_combine(const miso_attn_combine_params* p, void* stream) {
  if (p == nullptr || p->part_m == nullptr || p->part_l == nullptr || p->part_o == nullptr ||
      p->qg == nullptr || p->core == nullptr || p->n_splits == 0)
    return MISO_ERR_INVALID;
  k::attn_combine_kernel<64, true, 4><<<64, 64, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::AttnCombineParams*>(p));
  return launch_status();
}

int miso_attn_prefill(const miso_attn_prefill_params* p, void* stream) {
  if (p == nullptr || p->q == nullptr || p->qg == nullptr || p->k_cache == nullptr ||
      p->v_cache == nullptr || p->core == nullptr || uint64_t(p->pos0) + p->n > p->max_ctx ||
      !aligned16(p->q) || !aligned16(p->k_cache) || !aligned16(p->v_cache))
    return MISO_ERR_INVALID;
  if (p->n == 0)
    return MISO_OK;
  k::attn_prefill_kernel<256><<<k::attn_prefill_items(p->n), 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::AttnPrefillParams*>(p));
  return launch_status();
}

int miso_deltanet_step(const miso_deltanet_step_params* p, void* stream) {
  if (p == nullptr || p->qkv == nullptr || p->z == nullptr || p->a == nullptr ||
      p->b == nullptr || p->conv_w == nullptr || p->conv_in == nullptr ||
      p->conv_out == nullptr || p->ssm_a == nullptr || p->dt_bias == nullptr ||
      p->norm_w == nullptr || p->state == nullptr || p->out == nullptr || !aligned16(p->state))
    return MISO_ERR_INVALID;
  k::deltanet_step_kernel<256><<<32, 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::DeltaNetStepParams*>(p));
  return launch_status();
}

int miso_deltanet_seq(const miso_deltanet_seq_params* p, void* stream) {
  if (p == nullptr || p->qkv == nullptr || p->z == nullptr || p->a == nullptr ||
      p->b == nullptr || p->conv_w == nullptr || p->conv_in == nullptr ||
      p->conv_out == nullptr || p->ssm_a == nullptr || p->dt_bias == nullptr ||
      p->norm_w == nullptr || p->state == nullptr || p->out == nullptr || !aligned16(p->state))
    return MISO_ERR_INVALID;
  k::deltanet_seq_kernel<256><<<32, 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::DeltaNetSeqParams*>(p));
  return launch_status();
}

int miso_deltanet_seq_ckpt(const miso_deltanet_seq_params* p, float* state_ckpt,
                           float* conv_ckpt, void* stream) {
  if (p == nullptr || p->qkv == nullptr || p->z == nullptr || p->a == nullptr ||
      p->b == nullptr || p->conv_w == nullptr || p->conv_in == nullptr || p->ssm_a == nullptr ||
      p->dt_bias == nullptr || p->norm_w == nullptr || p->state == nullptr || p->out == nullptr ||
      state_ckpt == nullptr || conv_ckpt == nullptr || !aligned16(p->state) ||
      !aligned16(state_ckpt))
    return MISO_ERR_INVALID;
  k::deltanet_seq_ckpt_kernel<256><<<32, 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::DeltaNetSeqParams*>(p), state_ckpt, conv_ckpt);
  return launch_status();
}

int miso_deltanet_commit(const float* state_ckpt, const float* conv_ckpt, unsigned n,
                         unsigned k_accepted, float* state, float* conv_out, void* stream) {
  if (state_ckpt == nullptr || conv_ckpt == nullptr || state == nullptr || conv_out == nullptr ||
      k_accepted > n)
    return MISO_ERR_INVALID;
  if (k_accepted == 0)
    return 0;
  const std::size_t sf = std::size_t{32} * 128 * 128, cf = std::size_t{8192} * 3;
  cudaError_t e = cudaMemcpyAsync(state, state_ckpt + (k_accepted - 1) * sf, sf * sizeof(float),
                                  cudaMemcpyDeviceToDevice, as_stream(stream));
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(conv_out, conv_ckpt + (k_accepted - 1) * cf, cf * sizeof(float),
                        cudaMemcpyDeviceToDevice, as_stream(stream));
  return static_cast<int>(e);
}

int miso_deltanet_conv(const miso_deltanet_conv_params* p, void* stream) {
  if (p == nullptr || p->qkv == nullptr || p->conv_w == nullptr || p->conv_in == nullptr ||
      p->conv_out == nullptr || p->q == nullptr || p->k == nullptr || p->v == nullptr)
    return MISO_ERR_INVALID;
  k::deltanet_conv_kernel<<<32, 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::DeltaNetConvParams*>(p));
  return launch_status();
}

int miso_deltanet_norm(const miso_deltanet_conv_params* p, void* stream) {
  if (p == nullptr || p->q == nullptr || p->k == nullptr || p->a == nullptr || p->b == nullptr ||
      p->ssm_a == nullptr || p->dt_bias == nullptr || p->beta == nullptr ||
      p->log_a == nullptr || !aligned16(p->q) || !aligned16(p->k))
    return MISO_ERR_INVALID;
  k::deltanet_norm_kernel<<<64, 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::DeltaNetConvParams*>(p));
  return launch_status();
}

int miso_deltanet_chunk(const miso_deltanet_chunk_params* p, void* stream) {
  if (p == nullptr || p->q == nullptr || p->k == nullptr || p->v == nullptr ||
      p->beta == nullptr || p->log_a == nullptr || p->z == nullptr || p->norm_w == nullptr ||
      p->state == nullptr || p->out == nullptr || p->sk == nullptr || p->sq == nullptr ||
      !aligned16(p->q) || !aligned16(p->k) || !aligned16(p->sq) || !aligned16(p->z) ||
      !aligned16(p->out))
    return MISO_ERR_INVALID;
  k::deltanet_chunk_kernel<256><<<32, 256, 0, as_stream(stream)>>>(
      *reinterpret_cast<const k::DeltaNetChunkParams*>(p));
  return launch_status();
}

// ---- fast family ----------------------------------------------------------------------------

size_t miso_attn_decode_scratch_bytes(unsigned batch) {
  DeviceInfo* d = nullptr;
  if (device_info(&d) != MISO_OK)
    return 0;
  return decode_counter_bytes(batch) +
         size_t(2) * d->sms * miso::fast::decode::kPartFloats * sizeof(float);
}

int miso_attn_decode(const miso_attn_decode_params* p, void* scratch, size_t scratch_bytes,
                     void* stream) {
  namespace dec = miso::fast::decode;
  if (p == nullptr || p->q == nullptr || p->qg == nullptr || p->k_pool == nullptr ||
      p->v_pool == nullptr || p->kv_row == nullptr || p->lens == nullptr || p->core == nullptr ||
      p->batch == 0 || p->batch > unsigned(dec::kMaxBatch) || p->pool_rows == 0 ||
      p->pool_rows >= (uint64_t(1) << 31) || !aligned16(p->k_pool) || !aligned16(p->v_pool) ||
      (reinterpret_cast<uintptr_t>(p->q) & 7u) != 0 || scratch == nullptr ||
      (reinterpret_cast<uintptr_t>(scratch) & 255u) != 0)
    return MISO_ERR_INVALID;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != MISO_OK)
    return st;
  if ((st = tensor_map_encoder()) != MISO_OK)
    return st;
  const size_t need = decode_counter_bytes(p->batch) +
                      size_t(2) * d->sms * dec::kPartFloats * sizeof(float);
  if (scratch_bytes < need)
    return MISO_ERR_SCRATCH;
  CUtensorMap kmap, vmap;
  if ((st = kv_pool_map(&kmap, p->k_pool, p->pool_rows)) != MISO_OK ||
      (st = kv_pool_map(&vmap, p->v_pool, p->pool_rows)) != MISO_OK)
    return st;
  dec::Args a;
  a.q = p->q;
  a.qg = p->qg;
  a.kv_row = p->kv_row;
  a.lens = p->lens;
  a.core = p->core;
  a.counters = static_cast<int*>(scratch);
  a.parts = reinterpret_cast<float*>(static_cast<char*>(scratch) + decode_counter_bytes(p->batch));
  a.batch = p->batch;
  a.qg_stride = p->qg_stride;
  // The kernel returns every counter to zero, but a call whose bounded waits gave up does not:
  // start each call from zeroed counters so such a call cannot corrupt the next one.
  const cudaError_t e = cudaMemsetAsync(scratch, 0, size_t(2) * p->batch * sizeof(int),
                                        as_stream(stream));
  if (e != cudaSuccess)
    return static_cast<int>(e);
  const unsigned ctas = d->sms < int(dec::kMaxCtas) ? unsigned(d->sms) : dec::kMaxCtas;
  dec::decode_kernel<<<ctas, dec::kThreads, dec::kSmemBytes, as_stream(stream)>>>(kmap, vmap, a);
  return launch_status();
}

int miso_attn_prep_batched(const miso_attn_prep_batched_params* p, void* stream) {
  if (p == nullptr || p->qg == nullptr || p->k == nullptr || p->v == nullptr ||
      p->q_norm == nullptr || p->k_norm == nullptr || p->inv_freq == nullptr ||
      p->k_pool == nullptr || p->v_pool == nullptr || p->kv_row == nullptr ||
      p->lens == nullptr || p->q == nullptr || p->batch == 0 || p->batch > 65535 ||
      p->proj_stride % 4 != 0 || !aligned16(p->qg) || !aligned16(p->k) || !aligned16(p->v) ||
      !aligned16(p->q_norm) || !aligned16(p->k_norm) || !aligned16(p->q) ||
      !aligned16(p->k_pool) || !aligned16(p->v_pool))
    return MISO_ERR_INVALID;
  miso::fast::prep::Args a;
  a.qg = p->qg;
  a.k = p->k;
  a.v = p->v;
  a.q_norm = p->q_norm;
  a.k_norm = p->k_norm;
  a.inv_freq = p->inv_freq;
  a.k_pool = reinterpret_cast<__half*>(p->k_pool);
  a.v_pool = reinterpret_cast<__half*>(p->v_pool);
  a.kv_row = p->kv_row;
  a.lens = p->lens;
  a.q = p->q;
  a.batch = p->batch;
  a.proj_stride = p->proj_stride;
  a.eps = p->eps;
  miso::fast::prep::prep_batched_kernel<<<p->batch, miso::fast::prep::kThreads, 0,
                                           as_stream(stream)>>>(a);
  return launch_status();
}

}  // extern "C"

extern "C" {

int miso_attn_prep_batch_f16(const miso_attn_prep_batch_params* p, uint16_t* q_f16,
                             void* stream) {
  if (p == nullptr || q_f16 == nullptr || p->tok0.qg == nullptr || p->tok0.k == nullptr ||
      p->tok0.v == nullptr || p->tok0.q_norm == nullptr || p->tok0.k_norm == nullptr ||
      p->tok0.inv_freq == nullptr || p->tok0.k_cache == nullptr || p->tok0.v_cache == nullptr ||
      uint64_t(p->tok0.pos) + p->n > p->tok0.max_ctx || p->proj_stride % 4 != 0 ||
      !aligned16(p->tok0.qg) || !aligned16(p->tok0.k) || !aligned16(p->tok0.v) ||
      !aligned16(p->tok0.q_norm) || !aligned16(p->tok0.k_norm) || !aligned16(q_f16) ||
      !aligned16(p->tok0.k_cache) || !aligned16(p->tok0.v_cache))
    return MISO_ERR_INVALID;
  if (p->n == 0)
    return MISO_OK;
  miso::fast::prep::PrefillArgs a;
  a.qg = p->tok0.qg;
  a.k = p->tok0.k;
  a.v = p->tok0.v;
  a.q_norm = p->tok0.q_norm;
  a.k_norm = p->tok0.k_norm;
  a.inv_freq = p->tok0.inv_freq;
  a.k_cache = reinterpret_cast<__half*>(p->tok0.k_cache);
  a.v_cache = reinterpret_cast<__half*>(p->tok0.v_cache);
  a.q16 = reinterpret_cast<__half*>(q_f16);
  a.pos0 = p->tok0.pos;
  a.max_ctx = p->tok0.max_ctx;
  a.n = p->n;
  a.proj_stride = p->proj_stride;
  a.eps = p->tok0.eps;
  miso::fast::prep::prefill_prep_kernel<<<(p->n + miso::fast::prep::kPrepTokens - 1) /
                                              miso::fast::prep::kPrepTokens,
                                          miso::fast::prep::kThreads, 0, as_stream(stream)>>>(a);
  return launch_status();
}

int miso_attn_prefill_tc(const miso_attn_prefill_tc_params* p, void* stream) {
  namespace pf = miso::fast::prefill;
  if (p == nullptr || p->q == nullptr || p->qg == nullptr || p->k_cache == nullptr ||
      p->v_cache == nullptr || p->core == nullptr || p->n == 0 ||
      uint64_t(p->pos0) + p->n > p->max_ctx || uint64_t(p->pos0) + p->n >= (uint64_t(1) << 31) ||
      p->qg_stride % 4 != 0 || !aligned16(p->q) || !aligned16(p->qg) || !aligned16(p->k_cache) ||
      !aligned16(p->v_cache) || !aligned16(p->core))
    return MISO_ERR_INVALID;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != MISO_OK)
    return st;
  if ((st = tensor_map_encoder()) != MISO_OK)
    return st;
  CUtensorMap qmap, kmap, vmap;
  {
    const cuuint64_t dims[3] = {256, 16, p->n};
    const cuuint64_t strides[2] = {256 * 2, 16 * 256 * 2};
    const cuuint32_t box[3] = {64, 8, 16};
    if ((st = f16_map(&qmap, p->q, 3, dims, strides, box)) != MISO_OK)
      return st;
  }
  {
    const cuuint64_t dims[3] = {256, uint64_t(p->pos0) + p->n, 2};
    const cuuint64_t strides[2] = {256 * 2, uint64_t(p->max_ctx) * 256 * 2};
    const cuuint32_t kbox[3] = {64, pf::kBN, 1};  // 64 dims x one tile's keys
    const cuuint32_t vbox[3] = {64, 64, 1};       // 64 dims x 64 keys
    if ((st = f16_map(&kmap, p->k_cache, 3, dims, strides, kbox)) != MISO_OK ||
        (st = f16_map(&vmap, p->v_cache, 3, dims, strides, vbox)) != MISO_OK)
      return st;
  }
  pf::Args a;
  a.qg = p->qg;
  a.core = p->core;
  a.pos0 = p->pos0;
  a.n = p->n;
  a.qg_stride = p->qg_stride;
  a.n_qtiles = (p->n + pf::kTokens - 1) / pf::kTokens;
  pf::prefill_kernel<<<2 * a.n_qtiles, pf::kThreads, pf::kSmemBytes, as_stream(stream)>>>(
      qmap, kmap, vmap, a);
  return launch_status();
}

int miso_deltanet_step_batched(const miso_deltanet_step_batched_params* p, void* stream) {
  if (p == nullptr || p->qkv == nullptr || p->z == nullptr || p->a == nullptr ||
      p->b == nullptr || p->conv_w == nullptr || p->ssm_a == nullptr || p->dt_bias == nullptr ||
      p->norm_w == nullptr || p->conv_in == nullptr || p->conv_out == nullptr ||
      p->conv_in == p->conv_out || p->state == nullptr || p->out == nullptr || p->batch == 0 ||
      p->batch > 65535 || p->in_stride < 8192 || !aligned16(p->state) || !aligned16(p->out) ||
      !aligned16(p->norm_w) || !aligned16(p->conv_w))
    return MISO_ERR_INVALID;
  namespace ds = miso::fast::dnstep;
  ds::Args a;
  a.qkv = p->qkv;
  a.z = p->z;
  a.a = p->a;
  a.b = p->b;
  a.conv_w = p->conv_w;
  a.ssm_a = p->ssm_a;
  a.dt_bias = p->dt_bias;
  a.norm_w = p->norm_w;
  a.conv_in = p->conv_in;
  a.conv_out = p->conv_out;
  a.state = p->state;
  a.out = p->out;
  a.batch = p->batch;
  a.in_stride = p->in_stride;
  a.eps = p->eps;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != MISO_OK)
    return st;
  const unsigned units = p->batch * ds::kVHeads;
  const unsigned slots = unsigned(d->sms) * ds::kCtasPerSm;
  const unsigned ctas = units < slots ? units : slots;
  ds::step_batched_kernel<<<ctas, ds::kThreads, ds::kSmemBytes, as_stream(stream)>>>(a);
  return launch_status();
}

// Scratch of miso_deltanet_prefill_tc: the per-(V head, chunk) records front_kernel writes and
// chain_kernel reads, each part 1024-byte aligned (nc = ceil(n / 64)): Qg high and low parts and
// W [32][nc][64][128] fp16, U [32][nc][64][128] fp32, [Ks^T; Aqk] high and low parts
// [32][nc][192][64] fp16, e^(g_last) [32][nc] fp32.
struct DnScratch {
  size_t qgh, qgl, w, u, bh, bl, egl, total;
};

static DnScratch dn_scratch(unsigned n) {
  const size_t nc = (size_t(n) + 63) / 64;
  auto up = [](size_t x) { return (x + 1023) & ~size_t(1023); };
  DnScratch s;
  size_t o = 0;
  s.qgh = o, o += up(32 * nc * 64 * 128 * 2);
  s.qgl = o, o += up(32 * nc * 64 * 128 * 2);
  s.w = o, o += up(32 * nc * 64 * 128 * 2);
  s.u = o, o += up(32 * nc * 64 * 128 * 4);
  s.bh = o, o += up(32 * nc * 192 * 64 * 2);
  s.bl = o, o += up(32 * nc * 192 * 64 * 2);
  s.egl = o, o += up(32 * nc * 4);
  s.total = o;
  return s;
}

size_t miso_deltanet_prefill_tc_scratch_bytes(unsigned n) {
  return n == 0 ? 0 : dn_scratch(n).total;
}

}  // extern "C"

namespace {

// Stages of the tensor-core DeltaNet prefill: bit 0 = front_kernel (conv, norms and every
// state-independent product of each chunk; no state access), bit 1 = chain_kernel (the state
// recurrence and the pre-norm outputs, from the records bit 0 wrote), bit 2 = gate_kernel (the
// gated RMS norm of the outputs).
int dn_prefill_tc(const miso_deltanet_seq_params* p, void* scratch, size_t scratch_bytes,
                  void* stream, int stages) {
  namespace pf = miso::fast::dnpf;
  if (p == nullptr || p->qkv == nullptr || p->z == nullptr || p->a == nullptr ||
      p->b == nullptr || p->conv_w == nullptr || p->conv_in == nullptr ||
      p->conv_out == nullptr || p->conv_in == p->conv_out || p->ssm_a == nullptr ||
      p->dt_bias == nullptr || p->norm_w == nullptr || p->state == nullptr ||
      p->out == nullptr || p->n == 0 || p->n > (1u << 24) || p->qkv_stride % 4 != 0 ||
      p->qkv_stride < 8192 || p->zab_stride < 4160 || p->zab_stride % 4 != 0 ||
      !aligned16(p->qkv) || !aligned16(p->state) || !aligned16(p->conv_w) ||
      !aligned16(p->z) || !aligned16(p->norm_w) || !aligned16(p->out) || scratch == nullptr ||
      (reinterpret_cast<uintptr_t>(scratch) & 255u) != 0)
    return MISO_ERR_INVALID;
  const DnScratch L = dn_scratch(p->n);
  if (scratch_bytes < L.total)
    return MISO_ERR_SCRATCH;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != MISO_OK)
    return st;
  if ((st = tensor_map_encoder()) != MISO_OK)
    return st;
  char* base = static_cast<char*>(scratch);
  const unsigned nc = (p->n + 63) / 64;
  pf::Records rec;
  rec.qgh = reinterpret_cast<__half*>(base + L.qgh);
  rec.qgl = reinterpret_cast<__half*>(base + L.qgl);
  rec.w = reinterpret_cast<__half*>(base + L.w);
  rec.u = reinterpret_cast<float*>(base + L.u);
  rec.bh = reinterpret_cast<__half*>(base + L.bh);
  rec.bl = reinterpret_cast<__half*>(base + L.bl);
  rec.egl = reinterpret_cast<float*>(base + L.egl);
  cudaStream_t s = as_stream(stream);

  pf::FrontArgs fa;
  CUtensorMap qkvmap;
  if (stages & 1) {
    fa.qkv = p->qkv;
    fa.a = p->a;
    fa.b = p->b;
    fa.conv_w = p->conv_w;
    fa.conv_in = p->conv_in;
    fa.conv_out = p->conv_out;
    fa.ssm_a = p->ssm_a;
    fa.dt_bias = p->dt_bias;
    fa.rec = rec;
    fa.n = p->n;
    fa.nc = nc;
    fa.qkv_stride = p->qkv_stride;
    fa.zab_stride = p->zab_stride;
    fa.c0 = 0;
    fa.ahead = unsigned(d->sms);
    fa.per = nc;
    // Map over the q / k / v part of the projection rows (for the L2 prefetch of each chunk's
    // rows): 128 channels x 67 rows per box (a chunk and the three rows before it).
    const cuuint64_t dims[2] = {8192, p->n};
    const cuuint64_t strides[1] = {uint64_t(p->qkv_stride) * 4};
    const cuuint32_t box[2] = {128, 67};
    if ((st = f32_map(&qkvmap, p->qkv, dims, strides, box)) != MISO_OK)
      return st;
  }
  CUtensorMap qghmap, qglmap, wmap, umap, bhmap, blmap;
  pf::ChainArgs ca;
  pf::GateArgs ga;
  if (stages & 2) {
    {
      const cuuint64_t dims[2] = {128, uint64_t(32) * nc * 64};
      const cuuint64_t strides[1] = {128 * 2};
      const cuuint32_t box[2] = {64, 64};
      if ((st = f16_map(&qghmap, rec.qgh, 2, dims, strides, box)) != MISO_OK ||
          (st = f16_map(&qglmap, rec.qgl, 2, dims, strides, box)) != MISO_OK ||
          (st = f16_map(&wmap, rec.w, 2, dims, strides, box)) != MISO_OK)
        return st;
    }
    {
      const cuuint64_t dims[2] = {128, uint64_t(32) * nc * 64};
      const cuuint64_t strides[1] = {128 * 4};
      const cuuint32_t box[2] = {32, 64};
      if ((st = f32_map(&umap, rec.u, dims, strides, box)) != MISO_OK)
        return st;
    }
    {
      const cuuint64_t dims[2] = {64, uint64_t(32) * nc * 192};
      const cuuint64_t strides[1] = {64 * 2};
      const cuuint32_t box[2] = {64, 192};
      if ((st = f16_map(&bhmap, rec.bh, 2, dims, strides, box)) != MISO_OK ||
          (st = f16_map(&blmap, rec.bl, 2, dims, strides, box)) != MISO_OK)
        return st;
    }
    ca.egl = rec.egl;
    ca.state = p->state;
    ca.out = p->out;
    ca.n = p->n;
    ca.nc = nc;
  }
  ga.out = p->out;
  ga.z = p->z;
  ga.norm_w = p->norm_w;
  ga.zab_stride = p->zab_stride;
  ga.eps = p->eps;
  // Chunks [c0, c0 + cnt) of each stage.
  auto front = [&](cudaStream_t q, unsigned c0, unsigned cnt) {
    pf::FrontArgs f = fa;
    f.c0 = c0;
    pf::front_kernel<<<dim3(cnt, pf::kKHeads), pf::kFrontThreads, pf::kFrontSmemBytes, q>>>(
        qkvmap, f);
    return launch_status();
  };
  auto chain = [&](cudaStream_t q, unsigned c0, unsigned cnt) {
    pf::ChainArgs c = ca;
    c.c0 = c0;
    c.cnt = cnt;
    pf::chain_kernel<<<pf::kVHeads, pf::kChainThreads, pf::kChainSmemBytes, q>>>(
        qghmap, qglmap, wmap, umap, bhmap, blmap, c);
    return launch_status();
  };
  auto gate = [&](cudaStream_t q, unsigned c0, unsigned cnt) {
    pf::GateArgs g = ga;
    g.t0 = c0 * 64;
    g.n = (c0 + cnt) * 64 < p->n ? (c0 + cnt) * 64 : p->n;
    const unsigned rows = (g.n - g.t0) * pf::kVHeads, per_block = pf::kGateThreads / 32;
    const unsigned blocks = (rows + per_block - 1) / per_block;
    pf::gate_kernel<<<blocks < 8u * d->sms ? blocks : 8u * d->sms, pf::kGateThreads, 0, q>>>(g);
    return launch_status();
  };

  if (stages != 7 || nc <= kDnPieceChunks) {
    if ((stages & 1) && (st = front(s, 0, nc)) != MISO_OK)
      return st;
    if ((stages & 2) && (st = chain(s, 0, nc)) != MISO_OK)
      return st;
    if ((stages & 4) && (st = gate(s, 0, nc)) != MISO_OK)
      return st;
    return MISO_OK;
  }

  // Pipelined: the sequence in pieces of chunks; the front of piece k + 1 runs on the SMs the
  // chain of piece k leaves free (the chain uses one SM per V head), and the gate of piece k
  // overlaps both. Piece k's chain waits for its front and for piece k - 1's chain (stream order;
  // it carries the state), its gate for its chain.
  DnPipe* q = nullptr;
  if ((st = dn_pipe(&q)) != MISO_OK)
    return st;
  std::lock_guard<std::mutex> lock(q->mu);
  unsigned per = kDnPieceChunks;
  if ((nc + per - 1) / per + 1 > unsigned(kDnMaxPieces))
    per = (nc + kDnMaxPieces - 2) / (kDnMaxPieces - 1);
  // The first piece runs alone (nothing to overlap it with): a shorter one starts the chain
  // sooner.
  const unsigned first = kDnFirstPieceChunks < per ? kDnFirstPieceChunks : per;
  fa.ahead = unsigned(d->sms) > unsigned(pf::kVHeads) ? unsigned(d->sms) - pf::kVHeads : 1u;
  fa.per = per;
  auto ok = [](cudaError_t e) { return e == cudaSuccess ? MISO_OK : static_cast<int>(e); };
  if ((st = ok(cudaEventRecord(q->fork, s))) != MISO_OK ||
      (st = ok(cudaStreamWaitEvent(q->front, q->fork, 0))) != MISO_OK ||
      (st = ok(cudaStreamWaitEvent(q->chain, q->fork, 0))) != MISO_OK ||
      (st = ok(cudaStreamWaitEvent(q->gate, q->fork, 0))) != MISO_OK)
    return st;
  for (unsigned k = 0, c0 = 0, cnt = 0; c0 < nc; ++k, c0 += cnt) {
    const unsigned want = k == 0 ? first : per;
    cnt = nc - c0 < want ? nc - c0 : want;
    if ((st = front(q->front, c0, cnt)) != MISO_OK ||
        (st = ok(cudaEventRecord(q->front_done[k], q->front))) != MISO_OK ||
        (st = ok(cudaStreamWaitEvent(q->chain, q->front_done[k], 0))) != MISO_OK ||
        (st = chain(q->chain, c0, cnt)) != MISO_OK ||
        (st = ok(cudaEventRecord(q->chain_done[k], q->chain))) != MISO_OK ||
        (st = ok(cudaStreamWaitEvent(q->gate, q->chain_done[k], 0))) != MISO_OK ||
        (st = gate(q->gate, c0, cnt)) != MISO_OK)
      return st;
  }
  // Join: the caller's stream continues after the last gate (which follows every chain) and the
  // last front.
  if ((st = ok(cudaEventRecord(q->join_front, q->front))) != MISO_OK ||
      (st = ok(cudaEventRecord(q->join_gate, q->gate))) != MISO_OK ||
      (st = ok(cudaStreamWaitEvent(s, q->join_front, 0))) != MISO_OK ||
      (st = ok(cudaStreamWaitEvent(s, q->join_gate, 0))) != MISO_OK)
    return st;
  return MISO_OK;
}

}  // namespace

extern "C" {

int miso_deltanet_prefill_tc(const miso_deltanet_seq_params* p, void* scratch, size_t scratch_bytes,
                             void* stream) {
  return dn_prefill_tc(p, scratch, scratch_bytes, stream, 7);
}

int miso_deltanet_prefill_tc_front(const miso_deltanet_seq_params* p, void* scratch,
                                   size_t scratch_bytes, void* stream) {
  return dn_prefill_tc(p, scratch, scratch_bytes, stream, 1);
}

int miso_deltanet_prefill_tc_recur(const miso_deltanet_seq_params* p, void* scratch,
                                   size_t scratch_bytes, void* stream) {
  return dn_prefill_tc(p, scratch, scratch_bytes, stream, 2 | 4);
}

int miso_deltanet_prefill_tc_chain(const miso_deltanet_seq_params* p, void* scratch,
                                   size_t scratch_bytes, void* stream) {
  return dn_prefill_tc(p, scratch, scratch_bytes, stream, 2);
}

int miso_deltanet_prefill_tc_gate(const miso_deltanet_seq_params* p, void* scratch,
                                  size_t scratch_bytes, void* stream) {
  return dn_prefill_tc(p, scratch, scratch_bytes, stream, 4);
}

}  // extern "C"

// No-allocation variant of miso_attn_decode (its own file, same translation unit).
#include "decode_noalloc.cu"
