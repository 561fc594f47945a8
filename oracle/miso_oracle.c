/*
 * miso_oracle.c — CPU restatement of the reference's attention hot path (see miso_oracle.h).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library, used by tests/, smoke() and
 * bench.py's CPU baseline. Never linked into or called by the product path.
 *
 * Conventions: inputs are the fp32 / fp16 arrays the kernels read; all arithmetic is double.
 * Reference citations are to penta2himajin/miso (paths relative to its root).
 */
#define _GNU_SOURCE
#include "miso_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

enum { QH = 16, KVH = 2, D = 256, GROUP = 8, ROPE = 64 };
enum { DN_KH = 16, DN_VH = 32, DN_D = 128, DN_CH = 8192, DN_OUT = 4096, DN_C = 64 };

/* ---- small utilities ------------------------------------------------------------------------ */

double oracle_half_to_double(uint16_t h) {
  const int sign = (h >> 15) & 1, exp = (h >> 10) & 31, man = h & 1023;
  double v;
  if (exp == 0)
    v = ldexp((double)man, -24); /* subnormal: man * 2^-24 */
  else if (exp == 31)
    v = man ? NAN : INFINITY;
  else
    v = ldexp((double)(man | 1024), exp - 25);
  return sign ? -v : v;
}

/* Every binary16 value as a double, built once (exact: the same values as
 * oracle_half_to_double), so the attention loops index a table instead of decoding each element. */
static double g_half[65536];
static pthread_once_t g_half_once = PTHREAD_ONCE_INIT;

static void half_table_init(void) {
  for (unsigned h = 0; h < 65536; ++h)
    g_half[h] = oracle_half_to_double((uint16_t)h);
}

static const double* half_table(void) {
  pthread_once(&g_half_once, half_table_init);
  return g_half;
}

int oracle_cpu_count(void) {
  const long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

typedef void (*work_fn)(void* ctx, size_t item);

typedef struct {
  work_fn fn;
  void* ctx;
  size_t n;
  size_t next; /* atomic */
} pool_t;

static void* pool_worker(void* arg) {
  pool_t* p = (pool_t*)arg;
  for (;;) {
    const size_t i = __atomic_fetch_add(&p->next, 1, __ATOMIC_RELAXED);
    if (i >= p->n)
      break;
    p->fn(p->ctx, i);
  }
  return NULL;
}

/* Runs fn(ctx, i) for i in [0, n) on up to `threads` threads (<= 0: all online CPUs). */
static void parallel_for(size_t n, int threads, work_fn fn, void* ctx) {
  if (threads <= 0)
    threads = oracle_cpu_count();
  if ((size_t)threads > n)
    threads = (int)n;
  pool_t p = {fn, ctx, n, 0};
  if (threads <= 1) {
    pool_worker(&p);
    return;
  }
  pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  int started = 0;
  for (int t = 0; t < threads; ++t)
    if (pthread_create(&tid[t], NULL, pool_worker, &p) == 0)
      ++started;
  if (started == 0)
    pool_worker(&p);
  for (int t = 0; t < started; ++t)
    pthread_join(tid[t], NULL);
  free(tid);
}

static double sigmoid(double x) { return 1.0 / (1.0 + exp(-x)); }
static double silu(double x) { return x / (1.0 + exp(-x)); }
/* softplus with the reference's linear branch above 20 (kernels/deltanet_step.hpp:46-48). */
static double softplus(double x) { return x > 20.0 ? x : log1p(exp(x)); }

/* ---- attention ------------------------------------------------------------------------------ */

/* kernels/attention_decode.hpp:95-115 */
unsigned oracle_attn_n_splits(unsigned len, unsigned max_splits) {
  const unsigned subs = (len + 31) / 32;
  if (subs == 0)
    return 1;
  unsigned per = 6, n = (subs + per - 1) / per;
  if (n > max_splits) {
    per = (subs + max_splits - 1) / max_splits;
    n = (subs + per - 1) / per;
  } else if (n < 16 && max_splits >= 16) {
    const unsigned target = subs < 16 ? subs : 16;
    if (n < target) {
      per = (subs + target - 1) / target;
      n = (subs + per - 1) / per;
    }
  }
  return n;
}

/* One row of the prep: RMSNorm with weight, then NEOX rotation of dims < 64
 * (kernels/attention_decode.hpp:51-62). The angle is the fp32 product pos * inv_freq[i], as the
 * kernel forms it; sin / cos are then evaluated in double. */
static void prep_row(const float* x, const float* w, const float* inv_freq, unsigned pos,
                     float eps, double* y) {
  double ss = 0.0;
  for (int d = 0; d < D; ++d)
    ss += (double)x[d] * x[d];
  const double r = 1.0 / sqrt(ss / D + eps);
  double n[D];
  for (int d = 0; d < D; ++d)
    n[d] = x[d] * r * w[d];
  for (int d = 0; d < D; ++d)
    y[d] = n[d];
  for (int i = 0; i < ROPE / 2; ++i) {
    const float ang = (float)pos * inv_freq[i];
    const double c = cos((double)ang), s = sin((double)ang);
    y[i] = n[i] * c - n[i + ROPE / 2] * s;
    y[i + ROPE / 2] = n[i + ROPE / 2] * c + n[i] * s;
  }
}

void oracle_attn_prep(const float* qg, const float* k, const float* v, const float* q_norm,
                      const float* k_norm, const float* inv_freq, unsigned pos, float eps,
                      double* q_out, double* k_out, double* v_out) {
  for (int h = 0; h < QH; ++h)
    prep_row(qg + h * 2 * D, q_norm, inv_freq, pos, eps, q_out + h * D);
  for (int h = 0; h < KVH; ++h) {
    prep_row(k + h * D, k_norm, inv_freq, pos, eps, k_out + h * D);
    for (int d = 0; d < D; ++d)
      v_out[h * D + d] = v[h * D + d];
  }
}

/* softmax(q . K^T / 16) V * sigmoid(gate) for one query row over keys [0, len) of K/V rows
 * (tests/test_attn_splitk.hip:153-169). */
static void attend_row(const float* q, const float* gate, const uint16_t* K, const uint16_t* V,
                       unsigned len, double* s, double* out) {
  if (len == 0) {
    for (int e = 0; e < D; ++e)
      out[e] = 0.0;
    return;
  }
  const double* H = half_table();
  double mx = -INFINITY;
  for (unsigned j = 0; j < len; ++j) {
    double dot = 0.0;
    const uint16_t* kr = K + (size_t)j * D;
    for (int e = 0; e < D; ++e)
      dot += (double)q[e] * H[kr[e]];
    s[j] = dot / 16.0;
    if (s[j] > mx)
      mx = s[j];
  }
  double l = 0.0;
  for (unsigned j = 0; j < len; ++j) {
    s[j] = exp(s[j] - mx);
    l += s[j];
  }
  for (int e = 0; e < D; ++e)
    out[e] = 0.0;
  for (unsigned j = 0; j < len; ++j) {
    const uint16_t* vr = V + (size_t)j * D;
    for (int e = 0; e < D; ++e)
      out[e] += s[j] * H[vr[e]];
  }
  for (int e = 0; e < D; ++e)
    out[e] = out[e] / l / (1.0 + exp(-(double)gate[e]));
}

typedef struct {
  const float *q, *qg;
  unsigned qg_stride;
  const uint16_t *k_pool, *v_pool;
  const int64_t* kv_row;
  const int32_t* lens;
  double* out;
} decode_ctx;

static void decode_item(void* vctx, size_t item) {
  const decode_ctx* c = (const decode_ctx*)vctx;
  const size_t b = item / QH;
  const int h = (int)(item % QH), kvh = h / GROUP;
  const unsigned len = c->lens[b] > 0 ? (unsigned)c->lens[b] : 0;
  const size_t row0 = (size_t)c->kv_row[2 * b + kvh];
  double* s = (double*)malloc(sizeof(double) * (len ? len : 1));
  attend_row(c->q + (b * QH + h) * D, c->qg + b * c->qg_stride + h * 2 * D + D,
             c->k_pool + row0 * D, c->v_pool + row0 * D, len, s, c->out + (b * QH + h) * D);
  free(s);
}

void oracle_attn_decode(unsigned batch, const float* q, const float* qg, unsigned qg_stride,
                        const uint16_t* k_pool, const uint16_t* v_pool, const int64_t* kv_row,
                        const int32_t* lens, double* out, int threads) {
  decode_ctx c = {q, qg, qg_stride, k_pool, v_pool, kv_row, lens, out};
  parallel_for((size_t)batch * QH, threads, decode_item, &c);
}

typedef struct {
  unsigned pos0;
  const float *q, *qg;
  unsigned qg_stride;
  const uint16_t *k_cache, *v_cache;
  unsigned max_ctx;
  const unsigned* rows;
  double* out;
} prefill_ctx;

static void prefill_item(void* vctx, size_t item) {
  const prefill_ctx* c = (const prefill_ctx*)vctx;
  const size_t r = item / QH;
  const int h = (int)(item % QH), kvh = h / GROUP;
  const size_t t = c->rows ? c->rows[r] : r;
  const unsigned seen = c->pos0 + (unsigned)t + 1;
  double* s = (double*)malloc(sizeof(double) * seen);
  attend_row(c->q + (t * QH + h) * D, c->qg + t * c->qg_stride + h * 2 * D + D,
             c->k_cache + (size_t)kvh * c->max_ctx * D, c->v_cache + (size_t)kvh * c->max_ctx * D,
             seen, s, c->out + (r * QH + h) * D);
  free(s);
}

void oracle_attn_prefill(unsigned n, unsigned pos0, const float* q, const float* qg,
                         unsigned qg_stride, const uint16_t* k_cache, const uint16_t* v_cache,
                         unsigned max_ctx, const unsigned* rows, unsigned n_rows, double* out,
                         int threads) {
  prefill_ctx c = {pos0, q, qg, qg_stride, k_cache, v_cache, max_ctx, rows, out};
  parallel_for((size_t)(rows ? n_rows : n) * QH, threads, prefill_item, &c);
}

/* kernels/attention_decode.hpp:238-303 (merge of split partials, gated). */
void oracle_attn_combine(const float* part_m, const float* part_l, const float* part_o,
                         const float* qg, unsigned n_splits, double* core) {
  for (int h = 0; h < QH; ++h) {
    const int kvh = h / GROUP, hl = h % GROUP;
    double M = -INFINITY;
    for (unsigned c = 0; c < n_splits; ++c) {
      const double m = part_m[((size_t)kvh * n_splits + c) * GROUP + hl];
      if (m > M)
        M = m;
    }
    for (int d = 0; d < D; ++d) {
      double L = 0.0, o = 0.0;
      for (unsigned c = 0; c < n_splits; ++c) {
        const size_t i = ((size_t)kvh * n_splits + c) * GROUP + hl;
        const double w = exp((double)part_m[i] - M);
        L += w * part_l[i];
        o += w * part_o[i * D + d];
      }
      core[h * D + d] = o / L / (1.0 + exp(-(double)qg[h * 2 * D + D + d]));
    }
  }
}

/* ---- Gated DeltaNet ------------------------------------------------------------------------- */

/* Causal 4-tap conv + SiLU of one channel: taps 0..2 on the history (oldest first), tap 3 on the
 * current input (kernels/deltanet_step.hpp:50-61). */
static double conv_silu(const float* w, const double* hist, double x) {
  return silu(w[0] * hist[0] + w[1] * hist[1] + w[2] * hist[2] + w[3] * x);
}

static void shift_hist(double* hist, double x) {
  hist[0] = hist[1];
  hist[1] = hist[2];
  hist[2] = x;
}

/* The delta-rule update of one V head for one token from normalised q, k and raw v
 * (kernels/deltanet_step.hpp:97-131): S = decay S; delta = beta (v - S^T k); S += k delta^T;
 * o = S^T q; out = o * rsqrt(mean(o^2) + eps) * norm_w * SiLU(z). */
static void delta_rule(double* S, const double* q, const double* k, const double* v, double beta,
                       double decay, const float* norm_w, const float* z, float eps, double* out) {
  double kv[DN_D], o[DN_D];
  for (int vi = 0; vi < DN_D; ++vi)
    kv[vi] = 0.0;
  for (int kk = 0; kk < DN_D; ++kk) {
    double* row = S + (size_t)kk * DN_D;
    for (int vi = 0; vi < DN_D; ++vi) {
      row[vi] *= decay;
      kv[vi] += row[vi] * k[kk];
    }
  }
  double delta[DN_D];
  for (int vi = 0; vi < DN_D; ++vi) {
    delta[vi] = (v[vi] - kv[vi]) * beta;
    o[vi] = 0.0;
  }
  for (int kk = 0; kk < DN_D; ++kk) {
    double* row = S + (size_t)kk * DN_D;
    for (int vi = 0; vi < DN_D; ++vi) {
      row[vi] += k[kk] * delta[vi];
      o[vi] += row[vi] * q[kk];
    }
  }
  double ss = 0.0;
  for (int vi = 0; vi < DN_D; ++vi)
    ss += o[vi] * o[vi];
  const double r = 1.0 / sqrt(ss / DN_D + eps);
  for (int vi = 0; vi < DN_D; ++vi)
    out[vi] = o[vi] * r * norm_w[vi] * silu(z[vi]);
}

/* L2 normalisation with the 1e-6 inside the root (kernels/deltanet_step.hpp:91-93). */
static void l2norm(double* x, double extra) {
  double ss = 0.0;
  for (int i = 0; i < DN_D; ++i)
    ss += x[i] * x[i];
  const double r = extra / sqrt(ss + 1e-6);
  for (int i = 0; i < DN_D; ++i)
    x[i] *= r;
}

typedef struct {
  const float *qkv, *z, *a, *b, *conv_w;
  double* conv;
  const float *ssm_a, *dt_bias, *norm_w;
  double* state;
  double* out;
  float eps;
  double* y; /* [batch][8192] conv outputs */
} step_ctx;

static void step_conv_item(void* vctx, size_t bi) {
  const step_ctx* c = (const step_ctx*)vctx;
  for (int ch = 0; ch < DN_CH; ++ch) {
    double* hist = c->conv + (bi * DN_CH + ch) * 3;
    const double x = c->qkv[bi * DN_CH + ch];
    c->y[bi * DN_CH + ch] = conv_silu(c->conv_w + 4 * ch, hist, x);
  }
}

static void step_head_item(void* vctx, size_t item) {
  const step_ctx* c = (const step_ctx*)vctx;
  const size_t bi = item / DN_VH;
  const int h = (int)(item % DN_VH), kh = h % DN_KH;
  const double* y = c->y + bi * DN_CH;
  double q[DN_D], k[DN_D], v[DN_D];
  for (int i = 0; i < DN_D; ++i) {
    q[i] = y[kh * DN_D + i];
    k[i] = y[DN_KH * DN_D + kh * DN_D + i];
    v[i] = y[2 * DN_KH * DN_D + h * DN_D + i];
  }
  l2norm(q, 1.0 / sqrt((double)DN_D));
  l2norm(k, 1.0);
  const double beta = sigmoid(c->b[bi * DN_VH + h]);
  const double decay = exp(c->ssm_a[h] * softplus((double)c->a[bi * DN_VH + h] + c->dt_bias[h]));
  delta_rule(c->state + (bi * DN_VH + h) * DN_D * DN_D, q, k, v, beta, decay, c->norm_w,
             c->z + bi * DN_OUT + h * DN_D, c->eps, c->out + bi * DN_OUT + h * DN_D);
}

void oracle_deltanet_step(unsigned batch, const float* qkv, const float* z, const float* a,
                          const float* b, const float* conv_w, double* conv, const float* ssm_a,
                          const float* dt_bias, const float* norm_w, double* state, double* out,
                          float eps, int threads) {
  double* y = (double*)malloc(sizeof(double) * batch * DN_CH);
  step_ctx c = {qkv, z, a, b, conv_w, conv, ssm_a, dt_bias, norm_w, state, out, eps, y};
  parallel_for(batch, threads, step_conv_item, &c);
  parallel_for((size_t)batch * DN_VH, threads, step_head_item, &c);
  for (size_t i = 0; i < (size_t)batch * DN_CH; ++i)
    shift_hist(conv + i * 3, qkv[i]);
  free(y);
}

typedef struct {
  unsigned n;
  const float* qkv;
  unsigned qkv_stride;
  const float *z, *a, *b;
  unsigned zab_stride;
  const float* conv_w;
  const double* conv0; /* history before the first token */
  const float *ssm_a, *dt_bias, *norm_w;
  double* state;
  double* out;
  float eps;
  const unsigned* heads; /* V heads to run (NULL: all DN_VH, item = head) */
  unsigned n_heads;      /* with heads: out is [n][n_heads][128] in list order */
} seq_ctx;

/* One V head over all n tokens; each head keeps private copies of its channels' histories. */
static void seq_head_item(void* vctx, size_t hh) {
  const seq_ctx* c = (const seq_ctx*)vctx;
  const int h = c->heads ? (int)c->heads[hh] : (int)hh, kh = h % DN_KH;
  double* hist = (double*)malloc(sizeof(double) * 3 * DN_D * 3);
  const int chq = kh * DN_D, chk = DN_KH * DN_D + kh * DN_D, chv = 2 * DN_KH * DN_D + h * DN_D;
  for (int i = 0; i < DN_D; ++i)
    for (int j = 0; j < 3; ++j) {
      hist[(0 * DN_D + i) * 3 + j] = c->conv0[(chq + i) * 3 + j];
      hist[(1 * DN_D + i) * 3 + j] = c->conv0[(chk + i) * 3 + j];
      hist[(2 * DN_D + i) * 3 + j] = c->conv0[(chv + i) * 3 + j];
    }
  double q[DN_D], k[DN_D], v[DN_D];
  for (unsigned t = 0; t < c->n; ++t) {
    const float* x = c->qkv + (size_t)t * c->qkv_stride;
    for (int i = 0; i < DN_D; ++i) {
      q[i] = conv_silu(c->conv_w + 4 * (chq + i), hist + (0 * DN_D + i) * 3, x[chq + i]);
      k[i] = conv_silu(c->conv_w + 4 * (chk + i), hist + (1 * DN_D + i) * 3, x[chk + i]);
      v[i] = conv_silu(c->conv_w + 4 * (chv + i), hist + (2 * DN_D + i) * 3, x[chv + i]);
      shift_hist(hist + (0 * DN_D + i) * 3, x[chq + i]);
      shift_hist(hist + (1 * DN_D + i) * 3, x[chk + i]);
      shift_hist(hist + (2 * DN_D + i) * 3, x[chv + i]);
    }
    l2norm(q, 1.0 / sqrt((double)DN_D));
    l2norm(k, 1.0);
    const size_t zr = (size_t)t * c->zab_stride;
    const double beta = sigmoid(c->b[zr + h]);
    const double decay = exp(c->ssm_a[h] * softplus((double)c->a[zr + h] + c->dt_bias[h]));
    double* o = c->heads ? c->out + ((size_t)t * c->n_heads + hh) * DN_D
                         : c->out + (size_t)t * DN_OUT + h * DN_D;
    delta_rule(c->state + (size_t)h * DN_D * DN_D, q, k, v, beta, decay, c->norm_w,
               c->z + zr + h * DN_D, c->eps, o);
  }
  free(hist);
}

void oracle_deltanet_seq(unsigned n, const float* qkv, unsigned qkv_stride, const float* z,
                         const float* a, const float* b, unsigned zab_stride, const float* conv_w,
                         double* conv, const float* ssm_a, const float* dt_bias,
                         const float* norm_w, double* state, double* out, float eps, int threads) {
  double* conv0 = (double*)malloc(sizeof(double) * DN_CH * 3);
  memcpy(conv0, conv, sizeof(double) * DN_CH * 3);
  seq_ctx c = {n,     qkv,     qkv_stride, z,     a,   b,   zab_stride, conv_w, conv0,
               ssm_a, dt_bias, norm_w,     state, out, eps, NULL, 0};
  parallel_for(DN_VH, threads, seq_head_item, &c);
  /* Final history: the last three inputs of each channel (older history if n < 3). */
  for (int ch = 0; ch < DN_CH; ++ch) {
    double* hist = conv + (size_t)ch * 3;
    for (unsigned t = 0; t < n; ++t)
      shift_hist(hist, qkv[(size_t)t * qkv_stride + ch]);
  }
  free(conv0);
}

/* oracle_deltanet_seq for the listed V heads only (each head is independent of the others):
 * their state slices [h] are updated and their outputs written to out [n][n_heads][128] in list
 * order. The conv history is read, not updated. Same restatement as above
 * (kernels/deltanet_step.hpp:146-273). */
void oracle_deltanet_seq_heads(unsigned n, const float* qkv, unsigned qkv_stride, const float* z,
                               const float* a, const float* b, unsigned zab_stride,
                               const float* conv_w, const double* conv, const float* ssm_a,
                               const float* dt_bias, const float* norm_w, double* state,
                               double* out, float eps, const unsigned* heads, unsigned n_heads,
                               int threads) {
  seq_ctx c = {n,     qkv,     qkv_stride, z,     a,   b,   zab_stride, conv_w, conv,
               ssm_a, dt_bias, norm_w,     state, out, eps, heads, n_heads};
  parallel_for(n_heads, threads, seq_head_item, &c);
}

/* kernels/deltanet_chunk.hpp:41-112 */
void oracle_deltanet_prepare(unsigned n, const float* qkv, const float* a, const float* b,
                             const float* conv_w, double* conv, const float* ssm_a,
                             const float* dt_bias, double* q, double* k, double* v, double* beta,
                             double* log_a) {
  const int QK = DN_KH * DN_D;
  for (int ch = 0; ch < DN_CH; ++ch) {
    double* hist = conv + (size_t)ch * 3;
    for (unsigned t = 0; t < n; ++t) {
      const double x = qkv[(size_t)t * DN_CH + ch];
      const double y = conv_silu(conv_w + 4 * ch, hist, x);
      shift_hist(hist, x);
      if (ch < QK)
        q[(size_t)t * QK + ch] = y;
      else if (ch < 2 * QK)
        k[(size_t)t * QK + ch - QK] = y;
      else
        v[(size_t)t * DN_OUT + ch - 2 * QK] = y;
    }
  }
  for (unsigned t = 0; t < n; ++t) {
    for (int h = 0; h < DN_KH; ++h) {
      l2norm(q + ((size_t)t * DN_KH + h) * DN_D, 1.0 / sqrt((double)DN_D));
      l2norm(k + ((size_t)t * DN_KH + h) * DN_D, 1.0);
    }
    for (int h = 0; h < DN_VH; ++h) {
      const size_t i = (size_t)t * DN_VH + h;
      beta[i] = sigmoid(b[i]);
      log_a[i] = ssm_a[h] * softplus((double)a[i] + dt_bias[h]);
    }
  }
}

typedef struct {
  unsigned n;
  const double *q, *k, *v, *beta, *log_a;
  const float *z, *norm_w;
  double *state, *out;
  float eps;
} chunk_ctx;

static void chunk_head_item(void* vctx, size_t hh) {
  const chunk_ctx* c = (const chunk_ctx*)vctx;
  const int h = (int)hh, kh = h % DN_KH;
  double* S = c->state + (size_t)h * DN_D * DN_D;
  double* sk = (double*)malloc(sizeof(double) * DN_C * DN_D);
  double* sq = (double*)malloc(sizeof(double) * DN_C * DN_D);
  double* dl = (double*)malloc(sizeof(double) * DN_C * DN_D);
  double g[DN_C], kk[DN_C][DN_C], qk[DN_C][DN_C];
  for (unsigned t0 = 0; t0 < c->n; t0 += DN_C) {
    const unsigned C = c->n - t0 < DN_C ? c->n - t0 : DN_C;
    const double* K[DN_C];
    const double* Q[DN_C];
    for (unsigned i = 0; i < C; ++i) {
      K[i] = c->k + ((size_t)(t0 + i) * DN_KH + kh) * DN_D;
      Q[i] = c->q + ((size_t)(t0 + i) * DN_KH + kh) * DN_D;
    }
    double acc = 0.0;
    for (unsigned i = 0; i < C; ++i) {
      acc += c->log_a[(size_t)(t0 + i) * DN_VH + h];
      g[i] = acc;
    }
    for (unsigned i = 0; i < C; ++i)
      for (unsigned j = 0; j <= i; ++j) {
        double dk = 0.0, dq = 0.0;
        for (int e = 0; e < DN_D; ++e) {
          dk += K[i][e] * K[j][e];
          dq += Q[i][e] * K[j][e];
        }
        kk[i][j] = dk;
        qk[i][j] = dq;
      }
    for (unsigned i = 0; i < C; ++i)
      for (int vi = 0; vi < DN_D; ++vi) {
        double a1 = 0.0, a2 = 0.0;
        for (int r = 0; r < DN_D; ++r) {
          a1 += S[r * DN_D + vi] * K[i][r];
          a2 += S[r * DN_D + vi] * Q[i][r];
        }
        sk[i * DN_D + vi] = a1;
        sq[i * DN_D + vi] = a2;
      }
    for (unsigned i = 0; i < C; ++i) {
      const double bi = c->beta[(size_t)(t0 + i) * DN_VH + h], ei = exp(g[i]);
      const double* vv = c->v + ((size_t)(t0 + i) * DN_VH + h) * DN_D;
      for (int vi = 0; vi < DN_D; ++vi) {
        double x = bi * (vv[vi] - ei * sk[i * DN_D + vi]);
        for (unsigned j = 0; j < i; ++j)
          x -= bi * exp(g[i] - g[j]) * kk[i][j] * dl[j * DN_D + vi];
        dl[i * DN_D + vi] = x;
      }
    }
    for (unsigned i = 0; i < C; ++i) {
      double o[DN_D];
      const double ei = exp(g[i]);
      for (int vi = 0; vi < DN_D; ++vi) {
        double x = ei * sq[i * DN_D + vi];
        for (unsigned j = 0; j <= i; ++j)
          x += exp(g[i] - g[j]) * qk[i][j] * dl[j * DN_D + vi];
        o[vi] = x;
      }
      double ss = 0.0;
      for (int vi = 0; vi < DN_D; ++vi)
        ss += o[vi] * o[vi];
      const double r = 1.0 / sqrt(ss / DN_D + c->eps);
      const size_t row = ((size_t)(t0 + i) * DN_VH + h) * DN_D;
      for (int vi = 0; vi < DN_D; ++vi)
        c->out[row + vi] = o[vi] * r * c->norm_w[vi] * silu(c->z[row + vi]);
    }
    const double gl = g[C - 1], el = exp(gl);
    for (int r = 0; r < DN_D; ++r)
      for (int vi = 0; vi < DN_D; ++vi) {
        double add = 0.0;
        for (unsigned i = 0; i < C; ++i)
          add += exp(gl - g[i]) * K[i][r] * dl[i * DN_D + vi];
        S[r * DN_D + vi] = el * S[r * DN_D + vi] + add;
      }
  }
  free(sk);
  free(sq);
  free(dl);
}

void oracle_deltanet_chunk(unsigned n, const double* q, const double* k, const double* v,
                           const double* beta, const double* log_a, const float* z,
                           const float* norm_w, double* state, double* out, float eps,
                           int threads) {
  chunk_ctx c = {n, q, k, v, beta, log_a, z, norm_w, state, out, eps};
  parallel_for(DN_VH, threads, chunk_head_item, &c);
}
