/*
 * miso_cuda.h — C ABI of the B200 (sm_100a) attention hot path.
 *
 * Plain C: device pointers, sizes and an opaque stream. No C++ or framework types cross this
 * boundary, so it binds directly from C, C++ (the engine), Python ctypes or any other FFI.
 *
 * Conventions
 *   - Every pointer named in a params struct is a DEVICE pointer unless its comment says host.
 *   - `stream` is a cudaStream_t passed as void*; NULL is the legacy default stream.
 *   - Calls only enqueue work; none synchronises the host (except miso_device_status).
 *   - Return value: MISO_OK (0) on success; a negative MISO_ERR_* for a rejected argument (nothing
 *     was launched); a positive value is the cudaError_t reported by the launch.
 *   - The params structs are layout-identical to the reference's POD Params structs
 *     (miso::kernels::*Params in the drop-in headers; fp16 pointers appear here as uint16_t*),
 *     so a caller can pass a pointer to its existing Params object.
 *
 * Shapes are fixed by the model (Qwen3.5-MoE hybrid attention): 16 query heads, 2 KV heads,
 * head_dim 256, partial RoPE over the first 64 dims; DeltaNet 16 K heads, 32 V heads, d = 128.
 */
#ifndef MISO_CUDA_H
#define MISO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MISO_ATTN_Q_HEADS 16
#define MISO_ATTN_KV_HEADS 2
#define MISO_ATTN_DIM 256
#define MISO_ATTN_ROPE_DIM 64
#define MISO_ATTN_SUB_CHUNK 32 /* kAttnSubChunk, kernels/attention_decode.hpp:90 */
#define MISO_ATTN_Q_BLOCK 4    /* kAttnQBlock, kernels/attention_prefill.hpp:52 */
#define MISO_DN_K_HEADS 16
#define MISO_DN_V_HEADS 32
#define MISO_DN_DIM 128
#define MISO_DN_CHUNK 64 /* kDeltaChunk, kernels/deltanet_chunk.hpp:22 */

enum {
  MISO_OK = 0,
  MISO_ERR_INVALID = -1,   /* null pointer, size out of range or misaligned buffer */
  MISO_ERR_SCRATCH = -2,   /* scratch buffer smaller than the *_scratch_bytes() figure */
  MISO_ERR_NO_DEVICE = -3, /* no CUDA device, or not an sm_100 device */
  MISO_ERR_DRIVER = -4,    /* a driver entry point (tensor-map encoding) was unavailable */
  MISO_ERR_LIMIT = -5      /* request exceeds a fixed capacity (miso_attn_decode_noalloc) */
};

/* Device status word (miso_device_status): the first failure recorded on the device. Low byte:
 * MISO_STATUS_*; bits 8 and up: the kernel wait site that recorded it (0x11-0x13 batched decode,
 * 0x14 batched DeltaNet step, 0x20-0x21 tensor-core prefill, 0x30-0x31 tensor-core DeltaNet
 * prefill). */
enum { MISO_STATUS_OK = 0, MISO_STATUS_TIMEOUT = 1 };

/* ---------------------------------------------------------------------------------------------
 * Drop-in family: one entry point per reference __global__, same Params, same launch geometry
 * as the reference engine uses, same semantics.
 * ------------------------------------------------------------------------------------------- */

/* == miso::kernels::AttnPrepParams, kernels/attention_decode.hpp:19-31. */
typedef struct {
  const float* qg;       /* [16][512]: per head 256 query then 256 gate */
  const float* k;        /* [2][256] */
  const float* v;        /* [2][256] */
  const float* q_norm;   /* [256] (stores 1 + w) */
  const float* k_norm;   /* [256] */
  const float* inv_freq; /* [32] */
  uint16_t* k_cache;     /* fp16 [2][max_ctx][256] */
  uint16_t* v_cache;     /* fp16 [2][max_ctx][256] */
  float* q;              /* [16][256] normalised, rotated queries */
  unsigned pos, max_ctx;
  float eps;
} miso_attn_prep_params;

/* == miso::kernels::AttnPrepBatchParams, kernels/attention_decode.hpp:35-39. */
typedef struct {
  miso_attn_prep_params tok0;
  unsigned n;
  unsigned proj_stride;
} miso_attn_prep_batch_params;

/* == miso::kernels::AttnSplitParams, kernels/attention_decode.hpp:117-125. */
typedef struct {
  const float* q; /* [16][256] (unscaled) */
  const uint16_t* k_cache;
  const uint16_t* v_cache;
  float* part_m; /* [2][n_splits][8] */
  float* part_l; /* [2][n_splits][8] */
  float* part_o; /* [2][n_splits][8][256] */
  unsigned len, max_ctx, n_splits;
} miso_attn_split_params;

/* == miso::kernels::AttnCombineParams, kernels/attention_decode.hpp:238-245. */
typedef struct {
  const float* part_m;
  const float* part_l;
  const float* part_o;
  const float* qg; /* [16][512], gate half */
  float* core;     /* [16][256] */
  unsigned n_splits;
} miso_attn_combine_params;

/* == miso::kernels::AttnPrefillParams, kernels/attention_prefill.hpp:42-50. */
typedef struct {
  const float* q;  /* [n][16][256] normalised, rotated (unscaled) */
  const float* qg; /* gate at tok * qg_stride + head * 512 + 256 */
  const uint16_t* k_cache;
  const uint16_t* v_cache;
  float* core; /* [n][16][256] */
  unsigned pos0, n, max_ctx;
  unsigned qg_stride;
} miso_attn_prefill_params;

/* == miso::kernels::DeltaNetStepParams, kernels/deltanet_step.hpp:22-36. */
typedef struct {
  const float* qkv;     /* [8192]: q[2048] k[2048] v[4096] */
  const float* z;       /* [4096] */
  const float* a;       /* [32] */
  const float* b;       /* [32] */
  const float* conv_w;  /* [8192][4] */
  const float* conv_in; /* [8192][3] */
  float* conv_out;      /* [8192][3] */
  const float* ssm_a;   /* [32] */
  const float* dt_bias; /* [32] */
  const float* norm_w;  /* [128] */
  float* state;         /* [32][128 k][128 v] */
  float* out;           /* [4096] */
  float eps;
} miso_deltanet_step_params;

/* == miso::kernels::DeltaNetSeqParams, kernels/deltanet_step.hpp:146-163. */
typedef struct {
  const float* qkv; /* [n][qkv_stride] */
  const float* z;   /* [n][zab_stride] */
  const float* a;
  const float* b;
  const float* conv_w;
  const float* conv_in;
  float* conv_out;
  const float* ssm_a;
  const float* dt_bias;
  const float* norm_w;
  float* state;
  float* out; /* [n][4096] */
  unsigned n;
  float eps;
  unsigned zab_stride;
  unsigned qkv_stride;
} miso_deltanet_seq_params;

/* == miso::kernels::DeltaNetConvParams, kernels/deltanet_chunk.hpp:24-39. */
typedef struct {
  const float* qkv; /* [n][8192] */
  const float* a;   /* [n][32] */
  const float* b;   /* [n][32] */
  const float* conv_w;
  const float* conv_in;
  float* conv_out;
  const float* ssm_a;
  const float* dt_bias;
  float* q;     /* [n][16][128] */
  float* k;     /* [n][16][128] */
  float* v;     /* [n][32][128] */
  float* beta;  /* [n][32] */
  float* log_a; /* [n][32] */
  unsigned n;
} miso_deltanet_conv_params;

/* == miso::kernels::DeltaNetChunkParams, kernels/deltanet_chunk.hpp:114-128. */
typedef struct {
  const float* q;
  const float* k;
  const float* v;
  const float* beta;
  const float* log_a;
  const float* z; /* [n][4096] */
  const float* norm_w;
  float* state; /* [32][128][128] */
  float* out;   /* [n][4096] */
  float* sk;    /* [32][64][128] scratch */
  float* sq;    /* [32][64][128] scratch */
  unsigned n;
  float eps;
} miso_deltanet_chunk_params;

/* attn_n_splits, kernels/attention_decode.hpp:95-115 (host function, pure). */
unsigned miso_attn_n_splits(unsigned len, unsigned max_splits);
/* attn_prefill_items, kernels/attention_prefill.hpp:54-56 (host function, pure). */
unsigned miso_attn_prefill_items(unsigned n);

/* attn_prep_kernel<256><<<18, 256>>>, launched at src/engine/attention.hip:100. */
int miso_attn_prep(const miso_attn_prep_params* p, void* stream);
/* attn_prep_batch_kernel<256><<<n * 18, 256>>>, src/engine/attention.hip:140. */
int miso_attn_prep_batch(const miso_attn_prep_batch_params* p, void* stream);
/* attn_split_kernel<256><<<(n_splits, 2), 256>>>, src/engine/attention.hip:106. q, k_cache and
 * v_cache 16-byte aligned. */
int miso_attn_split(const miso_attn_split_params* p, void* stream);
/* attn_combine_kernel<64, true, 4><<<64, 64>>>, src/engine/attention.hip:109. */
int miso_attn_combine(const miso_attn_combine_params* p, void* stream);
/* attn_prefill_kernel<256><<<attn_prefill_items(n), 256>>>, src/engine/attention.hip:144. q,
 * k_cache and v_cache 16-byte aligned (MISO_ERR_INVALID otherwise). A token's result does not
 * depend on how the prompt is cut into calls (bitwise). */
int miso_attn_prefill(const miso_attn_prefill_params* p, void* stream);
/* deltanet_step_kernel<256><<<32, 256>>>, src/engine/deltanet.hip:79. */
int miso_deltanet_step(const miso_deltanet_step_params* p, void* stream);
/* deltanet_seq_kernel<256><<<32, 256>>>, src/engine/deltanet.hip:113. */
int miso_deltanet_seq(const miso_deltanet_seq_params* p, void* stream);

/* Speculative (multi-token prediction) verification of p->n draft tokens through a DeltaNet
 * layer, for the reference's planned commit / rollback of a variable number of accepted tokens
 * (docs/decisions/ADR_002-build-scope-numerics-ops.md D8). Same recurrence and outputs p->out as
 * miso_deltanet_seq, bit for bit, but p->state and p->conv_out are NOT written (p->conv_out may be
 * NULL); instead the state after token t goes to state_ckpt + t * 32*128*128 floats (16-byte
 * aligned) and the conv history after token t to conv_ckpt + t * 8192*3 floats.
 * miso_deltanet_commit then keeps the first k_accepted tokens: it copies checkpoint
 * k_accepted - 1 into state and conv_out (bitwise what miso_deltanet_seq over those tokens leaves;
 * flip the caller's conv parity as after miso_deltanet_seq), and for k_accepted == 0 changes
 * nothing. The KV side of a rollback is the cache length: set it to its pre-verification value
 * plus k_accepted. Errors: MISO_ERR_INVALID for NULL pointers or k_accepted > n. */
int miso_deltanet_seq_ckpt(const miso_deltanet_seq_params* p, float* state_ckpt,
                           float* conv_ckpt, void* stream);
int miso_deltanet_commit(const float* state_ckpt, const float* conv_ckpt, unsigned n,
                         unsigned k_accepted, float* state, float* conv_out, void* stream);
/* deltanet_conv_kernel<<<32, 256>>>, tests/test_deltanet_chunk.hip:82. */
int miso_deltanet_conv(const miso_deltanet_conv_params* p, void* stream);
/* deltanet_norm_kernel<<<64, 256>>>, tests/test_deltanet_chunk.hip:83. */
int miso_deltanet_norm(const miso_deltanet_conv_params* p, void* stream);
/* deltanet_chunk_kernel<256><<<32, 256>>>, tests/test_deltanet_chunk.hip:88. */
int miso_deltanet_chunk(const miso_deltanet_chunk_params* p, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Fast family: B200-native kernels with library-chosen geometry. No reference counterpart takes
 * a batch; each replaces a reference launch sequence as noted.
 * ------------------------------------------------------------------------------------------- */

/* Batched split-K decode over an fp16 KV pool. Replaces the attn_split_kernel +
 * attn_combine_kernel pair (src/engine/attention.hip:102-109) for `batch` sequences at once.
 * Sequence b, KV head h occupies pool rows [kv_row[2b+h], kv_row[2b+h] + lens[b]) of k_pool and
 * v_pool (a reference AttentionCache [2][max_ctx][256] is the case kv_row = {0, max_ctx}).
 *   core[b][h][d] = softmax(q[b][h] . K^T / 16) V [d] * sigmoid(qg[b * qg_stride + h*512 + 256 + d])
 * lens[b] == 0 gives core = 0. Work is divided evenly over the SMs by key tiles (stream-K); a
 * sequence cut across CTAs is merged by the last CTA to finish it, using `scratch`.
 * scratch: at least miso_attn_decode_scratch_bytes(batch) bytes, 256-byte aligned, any contents:
 * every call first zeroes the 2 * batch arrival counters at its start (an 8-byte-per-sequence
 * memset on `stream`, before the kernel), so the leftovers of an earlier call - including one
 * whose kernel gave up on a bounded wait and left counters set (miso_device_status then reports
 * MISO_STATUS_TIMEOUT) - do not reach the next call. Calls sharing one scratch buffer must not
 * overlap in time. Requires batch <= 1024, pool_rows < 2^31, 16-byte aligned pools. */
typedef struct {
  const float* q;         /* [batch][16][256] normalised, rotated queries (unscaled) */
  const float* qg;        /* gate of (b, h, d) at qg[b * qg_stride + h * 512 + 256 + d] */
  const uint16_t* k_pool; /* fp16 [pool_rows][256] */
  const uint16_t* v_pool; /* fp16 [pool_rows][256] */
  const int64_t* kv_row;  /* [batch][2] first pool row of each (sequence, KV head) */
  const int32_t* lens;    /* [batch] keys per sequence */
  float* core;            /* [batch][16][256] */
  uint64_t pool_rows;
  unsigned batch;
  unsigned qg_stride;
} miso_attn_decode_params;

size_t miso_attn_decode_scratch_bytes(unsigned batch);
int miso_attn_decode(const miso_attn_decode_params* p, void* scratch, size_t scratch_bytes,
                     void* stream);

/* miso_attn_decode for callers that cannot allocate device memory (no counterpart in the
 * reference, which is single-sequence and passes caller-owned scratch). Same parameters and
 * results as miso_attn_decode, without the scratch argument: the scratch is a fixed array inside
 * the library (2,643,968 bytes, present on every GPU that loads the library until exit). Limits:
 * batch <= 256 (MISO_ERR_LIMIT beyond). Allocates nothing. The first call on each device looks up
 * the array's address and should come before any stream capture (a failed lookup is returned as
 * that call's error and retried by the next call). All calls on a device share the array: calls
 * that overlap on the GPU race. */
int miso_attn_decode_noalloc(const miso_attn_decode_params* p, void* stream);

/* Batched decode prep: attn_prep_kernel (kernels/attention_decode.hpp:41-83) for `batch`
 * sequences, each at its own position pos = lens[b]; appends K/V to the pool rows kv_row[2b+h] +
 * pos and then sets lens[b] = pos + 1 (one CTA per sequence, so there is no race on lens[b]).
 * Token b's inputs: qg at qg + b*proj_stride ([16][512]), k at k + b*proj_stride ([2][256]),
 * v at v + b*proj_stride ([2][256]). */
typedef struct {
  const float* qg;
  const float* k;
  const float* v;
  const float* q_norm;
  const float* k_norm;
  const float* inv_freq;
  uint16_t* k_pool;
  uint16_t* v_pool;
  const int64_t* kv_row; /* [batch][2] */
  int32_t* lens;         /* [batch], read as the position, then incremented */
  float* q;              /* [batch][16][256] */
  unsigned batch;
  unsigned proj_stride;
  float eps;
} miso_attn_prep_batched_params;

int miso_attn_prep_batched(const miso_attn_prep_batched_params* p, void* stream);

/* Causal gated prefill on the tcgen05 tensor cores: the computation of attn_prefill_kernel
 * (kernels/attention_prefill.hpp:58-161, launched at src/engine/attention.hip:144) with fp16
 * queries, fp32 softmax and accumulation, library-chosen geometry. Accuracy: relative L2 ~1e-4
 * against the fp64 reference on N(0,1) data (fp16 rounding of Q and of the probabilities), where
 * the fp32-query drop-in kernel reaches 1e-5. Needs n >= 1, pos0 + n <= max_ctx, 16-byte aligned
 * q / caches / qg rows / core, qg_stride a multiple of 4. */
typedef struct {
  const uint16_t* q;       /* fp16 [n][16][256] normalised, rotated queries (unscaled) */
  const float* qg;         /* gate of (t, h, d) at qg[t * qg_stride + h * 512 + 256 + d] */
  const uint16_t* k_cache; /* fp16 [2][max_ctx][256], positions [0, pos0 + n) valid */
  const uint16_t* v_cache;
  float* core; /* [n][16][256] */
  unsigned pos0, n, max_ctx, qg_stride;
} miso_attn_prefill_tc_params;

int miso_attn_prefill_tc(const miso_attn_prefill_tc_params* p, void* stream);

/* attn_prep_batch_kernel (kernels/attention_prefill.hpp:20-40) with the queries written as fp16
 * to q_f16 [n][16][256] (the input of miso_attn_prefill_tc) instead of fp32 to p->tok0.q, which is
 * not used. K / V are appended to the fp16 cache exactly as by miso_attn_prep_batch. */
int miso_attn_prep_batch_f16(const miso_attn_prep_batch_params* p, uint16_t* q_f16, void* stream);

/* Batched Gated DeltaNet decode step: deltanet_step_kernel (kernels/deltanet_step.hpp:65-140,
 * launched at src/engine/deltanet.hip:79) for `batch` independent sequences in one launch.
 * Sequence b's inputs are the rows qkv / z / a / b + b * in_stride (8192 / 4096 / 32 / 32 values;
 * in_stride = 12352 for the engine's [qkv | z | a | b] projection rows); its conv history
 * [8192][3] at conv_in / conv_out + b * 24576 (double-buffered: conv_in != conv_out), its state
 * [32][128][128] at state + b * 524288 (updated in place), its output at out + b * 4096.
 * Weights (conv_w [8192][4], ssm_a, dt_bias [32], norm_w [128]) are shared. conv_w, state, out
 * and norm_w must be 16-byte aligned and in_stride at least 8192 (MISO_ERR_INVALID otherwise). */
typedef struct {
  const float* qkv;
  const float* z;
  const float* a;
  const float* b;
  const float* conv_w;
  const float* ssm_a;
  const float* dt_bias;
  const float* norm_w;
  const float* conv_in;
  float* conv_out;
  float* state;
  float* out;
  unsigned batch, in_stride;
  float eps;
} miso_deltanet_step_batched_params;

int miso_deltanet_step_batched(const miso_deltanet_step_batched_params* p, void* stream);

/* Gated DeltaNet prefill of n tokens on the tensor cores: the same inputs, outputs, conv history
 * hand-off and in-place state update as miso_deltanet_seq (deltanet_seq_kernel,
 * kernels/deltanet_step.hpp:146-273, launched at src/engine/deltanet.hip:112), computed with the
 * chunked gated delta rule (chunk 64; kernels/deltanet_chunk.hpp:3-9) instead of token by token.
 * Outputs agree with the recurrence to ~1e-4 relative (fp16 operands, fp32 accumulation and
 * state). Requires conv_in != conv_out, qkv, z, norm_w, out and state 16-byte aligned, qkv_stride
 * and zab_stride multiples of 4, and `scratch` (256-byte aligned) of at least
 * miso_deltanet_prefill_tc_scratch_bytes(n) bytes, which the call overwrites. For n > 2048 the
 * call runs the sequence in pieces (1024 tokens, then 2048 each) on three internal streams of the device (fork
 * from and join into `stream` by events, so the call stays ordered on `stream`); the first such
 * call on a device creates those streams and events, so it should come before any stream
 * capture, and calls from several host threads are serialised while they enqueue. */
size_t miso_deltanet_prefill_tc_scratch_bytes(unsigned n);
int miso_deltanet_prefill_tc(const miso_deltanet_seq_params* p, void* scratch, size_t scratch_bytes,
                             void* stream);

/* The same prefill in two calls, for callers that run the part that does not depend on the state
 * ahead of the state's arrival (a context-parallel wavefront receives the state of a segment from
 * the rank before it). _front: the conv, the per-chunk tiles and the conv history; reads qkv, a,
 * b, conv_w, conv_in, ssm_a, dt_bias, writes conv_out and the scratch, and neither reads nor
 * writes the state. _recur: the recurrence; reads the scratch written by a _front call with the
 * same p->n and the same scratch, and z, norm_w and the state; writes the state (in place) and
 * out. _front followed by _recur equals miso_deltanet_prefill_tc bit for bit. */
int miso_deltanet_prefill_tc_front(const miso_deltanet_seq_params* p, void* scratch,
                                   size_t scratch_bytes, void* stream);
int miso_deltanet_prefill_tc_recur(const miso_deltanet_seq_params* p, void* scratch,
                                   size_t scratch_bytes, void* stream);

/* The two parts of _recur, for callers whose next step needs only the state: _chain runs the
 * recurrence (reads the scratch of a _front call, z is not read; writes the state and the
 * pre-norm outputs to out), _gate then applies the gated RMS norm to out in place (reads z and
 * norm_w; scratch is only validated). _chain followed by _gate equals _recur bit for bit. */
int miso_deltanet_prefill_tc_chain(const miso_deltanet_seq_params* p, void* scratch,
                                   size_t scratch_bytes, void* stream);
int miso_deltanet_prefill_tc_gate(const miso_deltanet_seq_params* p, void* scratch,
                                  size_t scratch_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Library state
 * ------------------------------------------------------------------------------------------- */

/* Reads (and if reset != 0 clears) the device status word of the current device. Synchronises
 * the device. A kernel that gave up on a bounded wait records MISO_STATUS_TIMEOUT there. */
int miso_device_status(int reset, int* status);

/* Version string of the built library. */
const char* miso_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MISO_CUDA_H */
