/*
 * miso_oracle.h — CPU restatement of the reference's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This code is the checker for the CUDA library: it is called by
 * tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline / reference arm, never by the
 * product path. Everything is computed in double precision from the fp32 / fp16 inputs the GPU
 * kernels read, following the reference's scalar references and kernel formulas (each function
 * cites the reference file:line it restates).
 *
 * Threading: functions taking `threads` split independent (sequence, head) or (token, head)
 * units over that many POSIX threads (threads <= 0 means one per online CPU).
 */
#ifndef MISO_ORACLE_H
#define MISO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 bits -> double (exact). */
double oracle_half_to_double(uint16_t h);

/* attn_n_splits policy, kernels/attention_decode.hpp:95-115. */
unsigned oracle_attn_n_splits(unsigned len, unsigned max_splits);

/* Decode prep, kernels/attention_decode.hpp:41-71 with inv_freq per src/engine/attention.hip:65-69:
 * per head x <- x * rsqrt(mean(x^2) + eps) * w (q_norm for the 16 query heads, k_norm for the 2
 * KV heads), then NEOX rotation of dims [0, 64) by angle fp32(pos * inv_freq[i]).
 * q_out [16][256], k_out [2][256] (pre-cache-rounding), v_out [2][256] (= v). */
void oracle_attn_prep(const float* qg, const float* k, const float* v, const float* q_norm,
                      const float* k_norm, const float* inv_freq, unsigned pos, float eps,
                      double* q_out, double* k_out, double* v_out);

/* Batched split-K decode reference, tests/test_attn_splitk.hip:150-173, for `batch` sequences:
 * out[b][h][e] = (sum_j e^(s_j - max) v_j[e]) / (sum_j e^(s_j - max)) / (1 + e^(-gate)),
 * s_j = q[b][h] . k_j / 16, K/V rows of (b, kvh) at pool row kv_row[2b + kvh] + j, j < lens[b].
 * lens[b] == 0 gives out = 0. Gate of (b, h, e) at qg[b * qg_stride + h * 512 + 256 + e]. */
void oracle_attn_decode(unsigned batch, const float* q, const float* qg, unsigned qg_stride,
                        const uint16_t* k_pool, const uint16_t* v_pool, const int64_t* kv_row,
                        const int32_t* lens, double* out, int threads);

/* Causal prefill reference, tests/test_attn_splitk.hip:237-266: token t (position pos0 + t) sees
 * keys [0, pos0 + t] of a [2][max_ctx][256] fp16 cache. q [n][16][256], gate at
 * qg[t * qg_stride + h * 512 + 256 + e]. If rows != NULL only the n_rows listed tokens are
 * computed (out then holds n_rows x 16 x 256 values in list order); else all n tokens. */
void oracle_attn_prefill(unsigned n, unsigned pos0, const float* q, const float* qg,
                         unsigned qg_stride, const uint16_t* k_cache, const uint16_t* v_cache,
                         unsigned max_ctx, const unsigned* rows, unsigned n_rows, double* out,
                         int threads);

/* Partial-merge of split-K results, the combine of kernels/attention_decode.hpp:238-303, in
 * double: core[h][d] = (sum_c w_c o_c[d]) / (sum_c w_c l_c) / (1 + e^(-gate)), w_c = e^(m_c - M). */
void oracle_attn_combine(const float* part_m, const float* part_l, const float* part_o,
                         const float* qg, unsigned n_splits, double* core);

/* One Gated DeltaNet decode step for `batch` independent sequences,
 * kernels/deltanet_step.hpp:3-13 (formulas) and :50-135 (operation order). Per sequence b:
 * qkv [8192], z [4096], a/b [32] at b * {8192, 4096, 32, 32}; conv history [8192][3] and state
 * [32][128][128] (k-major) at b * {24576, 524288}, updated in place (double); out [4096] at
 * b * 4096. Shared weights conv_w [8192][4], ssm_a, dt_bias [32], norm_w [128]. */
void oracle_deltanet_step(unsigned batch, const float* qkv, const float* z, const float* a,
                          const float* b, const float* conv_w, double* conv, const float* ssm_a,
                          const float* dt_bias, const float* norm_w, double* state, double* out,
                          float eps, int threads);

/* n tokens of the same recurrence for one sequence (kernels/deltanet_step.hpp:142-273):
 * qkv row t at qkv + t * qkv_stride, z / a / b rows at + t * zab_stride. out [n][4096]. */
void oracle_deltanet_seq(unsigned n, const float* qkv, unsigned qkv_stride, const float* z,
                         const float* a, const float* b, unsigned zab_stride, const float* conv_w,
                         double* conv, const float* ssm_a, const float* dt_bias,
                         const float* norm_w, double* state, double* out, float eps, int threads);

/* oracle_deltanet_seq restricted to the n_heads V heads listed in `heads` (the heads do not
 * interact): updates their state slices and writes their outputs to out [n][n_heads][128] (list
 * order); the conv history is read, not updated. */
void oracle_deltanet_seq_heads(unsigned n, const float* qkv, unsigned qkv_stride, const float* z,
                               const float* a, const float* b, unsigned zab_stride,
                               const float* conv_w, const double* conv, const float* ssm_a,
                               const float* dt_bias, const float* norm_w, double* state,
                               double* out, float eps, const unsigned* heads, unsigned n_heads,
                               int threads);

/* Conv + SiLU + norm pass of the chunked form (kernels/deltanet_chunk.hpp:41-112): from qkv
 * [n][8192], a / b [n][32] produce q, k [n][16][128] (L2-normalised, q also / sqrt(128)),
 * v [n][32][128], beta and log_a [n][32]; conv history updated in place. */
void oracle_deltanet_prepare(unsigned n, const float* qkv, const float* a, const float* b,
                             const float* conv_w, double* conv, const float* ssm_a,
                             const float* dt_bias, double* q, double* k, double* v, double* beta,
                             double* log_a);

/* Chunked gated delta rule (chunk C = 64), kernels/deltanet_chunk.hpp:3-9, in double, from the
 * prepared q / k / v / beta / log_a; z [n][4096]; state [32][128][128] updated; out [n][4096]. */
void oracle_deltanet_chunk(unsigned n, const double* q, const double* k, const double* v,
                           const double* beta, const double* log_a, const float* z,
                           const float* norm_w, double* state, double* out, float eps,
                           int threads);

/* Online CPUs (for reporting the core count of a timed run). */
int oracle_cpu_count(void);

#ifdef __cplusplus
}
#endif

#endif /* MISO_ORACLE_H */
