/*
 * oracle.c -- CPU restatement of the reference token loop (TEST INFRASTRUCTURE ONLY).
 *
 * Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU legs as the checker and the
 * timed CPU baseline.  Nothing in the product library links or calls this file.
 * Every function cites the reference file:line it follows; see oracle.h for the summary
 * and for the statement that end-to-end parity is unpinned by the reference.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off; the reference's
 * `sum += a*b` loops are unfused on amd64, the platform whose evaluation this follows).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BOS_TOKEN 1 /* ane/stories/infer.go:10 */
#define EOS_TOKEN 2 /* ane/stories/infer.go:11 */

/* ------------------------------------------------------------------ rounding helpers */

float oracle_round_f16(float x) { return (float)(_Float16)x; }

float oracle_round_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) { /* inf / nan: keep (quiet nan) */
    if (u & 0x007fffffu) u |= 0x00400000u;
    u &= 0xffff0000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest even */
    u &= 0xffff0000u;
  }
  float r;
  memcpy(&r, &u, 4);
  return r;
}

static int mode_act(int mode) { /* 0: none, 1: fp16, 2: bf16 */
  switch (mode) {
    case ORACLE_F16: case ORACLE_W8A8_F16: return 1;
    case ORACLE_BF16: case ORACLE_W8A8_BF16: return 2;
    default: return 0;
  }
}
static int mode_int8(int mode) { return mode == ORACLE_W8A8_F16 || mode == ORACLE_W8A8_BF16; }

static inline float round_act(int act, float x) {
  return act == 1 ? oracle_round_f16(x) : (act == 2 ? oracle_round_bf16(x) : x);
}
static void round_vec(int act, float *v, int n) {
  if (!act) return;
  for (int i = 0; i < n; i++) v[i] = round_act(act, v[i]);
}

/* ------------------------------------------------------------------ threads */

static int g_threads = 0;
/* Test-only knob: 1 reverses the order of the PV sums in attention.  Used to measure how
 * far a correct implementation that merely sums in another order can drift. */
static int g_attn_reverse = 0;
void oracle_set_attn_reverse(int on) { g_attn_reverse = on; }
static int g_matvec_reverse = 0;
void oracle_set_matvec_reverse(int on) { g_matvec_reverse = on; }
void oracle_set_threads(int n) {
  g_threads = n;
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
}
int oracle_get_threads(void) {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------ building blocks */

/* ane/stories/infer.go:373-383 -- strict '>' so the first maximum wins. */
int oracle_argmax(const float *v, int n) {
  int best = 0;
  float bestv = v[0];
  for (int i = 1; i < n; i++)
    if (v[i] > bestv) { bestv = v[i]; best = i; }
  return best;
}

/* ane/stories/infer.go:301-311 -- float64 sum of squares, f32 rrms, x*rrms*w left to right.
 * eps is the float64 constant (Go: 1e-5). */
void oracle_rmsnorm(float *out, const float *x, const float *w, int n, double eps) {
  double sum = 0.0;
  for (int i = 0; i < n; i++) {
    double v = (double)x[i];
    sum += v * v;
  }
  float rrms = (float)(1.0 / sqrt(sum / (double)n + eps));
  for (int i = 0; i < n; i++) out[i] = x[i] * rrms * w[i];
}

/* ane/stories/infer.go:97-107 -- freq = pos / theta^(2i/hd) in float64, cos/sin -> f32. */
void oracle_rope_tables(int max_pos, int hd, double theta, float *cos_out, float *sin_out) {
  int half = hd / 2;
  for (int pos = 0; pos < max_pos; pos++)
    for (int i = 0; i < half; i++) {
      double freq = (double)pos / pow(theta, (double)(2 * i) / (double)hd);
      cos_out[pos * half + i] = (float)cos(freq);
      sin_out[pos * half + i] = (float)sin(freq);
    }
}

/* ane/stories/infer.go:328-345 */
void oracle_softmax_prefix(float *dst, const float *src, int n) {
  float mx = src[0];
  for (int i = 1; i < n; i++)
    if (src[i] > mx) mx = src[i];
  double sum = 0.0;
  for (int i = 0; i < n; i++) {
    float e = (float)exp((double)(src[i] - mx));
    dst[i] = e;
    sum += (double)e;
  }
  float inv = (float)(1.0 / sum);
  for (int i = 0; i < n; i++) dst[i] *= inv;
}

/* ane/stories/infer.go:324-326 */
float oracle_silu(float x) { return x / (1.0f + (float)exp((double)(-x))); }

/* bridge/ane_bridge.m:374-398, applied to one row (the reference applies it to a whole
 * tensor; per-row application is the W8A8 spec's per-channel / per-token granularity). */
static float quant_row(const float *x, int n, int8_t *q) {
  float max_abs = 0.0f;
  for (int i = 0; i < n; i++) {
    float a = x[i] < 0 ? -x[i] : x[i];
    if (a > max_abs) max_abs = a;
  }
  float scale = max_abs / 127.0f;
  if (scale == 0.0f) scale = 1.0f;
  for (int i = 0; i < n; i++) {
    float v = x[i] / scale;
    if (v > 127.0f) v = 127.0f;
    if (v < -128.0f) v = -128.0f;
    q[i] = (int8_t)(v + (v >= 0 ? 0.5f : -0.5f));
  }
  return scale;
}

void oracle_quant_rows(const float *x, int rows, int cols, int8_t *q, float *scales) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) scales[r] = quant_row(x + (size_t)r * cols, cols, q + (size_t)r * cols);
}

/* Sum of squares in the CUDA row kernel's order: the row is handled by T = n / (4*G)
 * threads (G = 2 float4 groups per thread when n >= 512, else 1); thread t owns the groups
 * starting at 4*t + 4*T*j (j = 0..G-1) and accumulates x*x in float64 (no fused
 * multiply-add) j-major, component-minor; each 32-thread warp combines its partials by an
 * xor butterfly (16, 8, 4, 2, 1); the warp totals are added in warp order. */
static double sumsq_lane_order(const float *x, int n) {
  int G = n >= 512 ? 2 : 1;
  int T = n / (4 * G);
  int W = (T + 31) / 32;
  double total = 0.0;
  for (int w = 0; w < W; w++) {
    double p[32];
    for (int l = 0; l < 32; l++) {
      int t = 32 * w + l;
      double acc = 0.0;
      if (t < T)
        for (int j = 0; j < G; j++)
          for (int c = 0; c < 4; c++) {
            double v = (double)x[4 * t + 4 * T * j + c];
            double sq = v * v;
            acc = acc + sq;
          }
      p[l] = acc;
    }
    for (int k = 16; k >= 1; k >>= 1) {
      double tt[32];
      for (int l = 0; l < 32; l++) tt[l] = p[l] + p[l ^ k];
      memcpy(p, tt, sizeof p);
    }
    total = w == 0 ? p[0] : total + p[0];
  }
  return total;
}

static float rrms_from_sumsq(double sum, int n, double eps) {
  return (float)(1.0 / sqrt(sum / (double)n + eps));
}

void oracle_norm_rows_lane_order(const float *x, const float *w, int rows, int cols, double eps,
                                 int round_mode, float *out) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    const float *xr = x + (size_t)r * cols;
    float rrms = rrms_from_sumsq(sumsq_lane_order(xr, cols), cols, eps);
    for (int i = 0; i < cols; i++) out[(size_t)r * cols + i] = round_act(round_mode, xr[i] * rrms * w[i]);
  }
}

void oracle_norm_quant_rows_lane_order(const float *x, const float *w, int rows, int cols,
                                       double eps, int8_t *q, float *scales) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    const float *xr = x + (size_t)r * cols;
    float rrms = rrms_from_sumsq(sumsq_lane_order(xr, cols), cols, eps);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)cols);
    for (int i = 0; i < cols; i++) tmp[i] = xr[i] * rrms * w[i];
    scales[r] = quant_row(tmp, cols, q + (size_t)r * cols);
    free(tmp);
  }
}

void oracle_gemm_i8(const int8_t *A, const int8_t *B, int M, int N, int K, int32_t *C) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int m = 0; m < M; m++)
    for (int n = 0; n < N; n++) {
      int32_t acc = 0;
      const int8_t *a = A + (size_t)m * K, *b = B + (size_t)n * K;
      for (int k = 0; k < K; k++) acc += (int32_t)a[k] * (int32_t)b[k];
      C[(size_t)m * N + n] = acc;
    }
}

float oracle_dequant(int32_t acc, float sa, float sw) { return ((float)acc * sa) * sw; }

/* ------------------------------------------------------------------ model */

typedef struct {
  /* F32 / F16 / BF16: dense float rows (rounded in the emulation modes) */
  float *f;          /* owned copy, or NULL when borrowed */
  const float *fp;   /* the rows used */
  /* W8A8 */
  int8_t *q;
  float *s;          /* per output row */
  int rows, cols;
} mat_t;

typedef struct {
  mat_t wq, wk, wv, wo, w1, w2, w3;
  const float *rms_att, *rms_ffn, *q_norm, *k_norm;
} layer_t;

struct oracle_model {
  oracle_config c;
  int act, i8;
  int q_dim, kv_dim, group;
  float *embed_r;          /* rounded embed (emulation) or NULL */
  const float *embed;      /* [vocab, dim] */
  const float *lm_head;    /* [vocab, dim] */
  float *lm_head_r;
  const float *rms_final;
  layer_t *layers;
  float *rope_cos, *rope_sin;
  float resid_scale; /* 0: x + branch (stories); else x + resid_scale * branch (storiesane) */
  int silu_form;     /* 0: h1 / (1 + exp(-h1)); 1: h1 * f32(1 / (1 + exp(-h1))) (storiesane) */
};

/* Select the storiesane CPU forward's arithmetic (ane/storiesane/engine.go:804-842). */
void oracle_model_set_storiesane(oracle_model *m, int on) {
  m->resid_scale = on ? (float)(1.0 / sqrt(2.0 * (double)m->c.n_layers)) : 0.0f;
  m->silu_form = on ? 1 : 0;
}

struct oracle_seq {
  const oracle_model *m;
  float *kcache, *vcache; /* [layer][pos][kv_dim] */
  float *x, *xn, *q, *k, *v, *att, *x2, *h1, *h3, *g, *y, *logits;
  int8_t *qa;
};

static void mat_init(mat_t *mt, const float *src, int rows, int cols, int act, int i8) {
  memset(mt, 0, sizeof *mt);
  mt->rows = rows;
  mt->cols = cols;
  size_t n = (size_t)rows * cols;
  if (i8) {
    mt->q = (int8_t *)malloc(n);
    mt->s = (float *)malloc(sizeof(float) * (size_t)rows);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) mt->s[r] = quant_row(src + (size_t)r * cols, cols, mt->q + (size_t)r * cols);
  } else if (act) {
    mt->f = (float *)malloc(sizeof(float) * n);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) mt->f[i] = round_act(act, src[i]);
    mt->fp = mt->f;
  } else {
    mt->fp = src;
  }
}

static void mat_free(mat_t *mt) {
  free(mt->f);
  free(mt->q);
  free(mt->s);
}

oracle_model *oracle_model_new(const oracle_config *cfg, const oracle_weights_f32 *w) {
  if (!cfg || !w || !w->embed || !w->layers || !w->rms_final) return NULL;
  const oracle_config *c = cfg;
  if (c->dim <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 || c->head_dim <= 1 ||
      c->vocab <= 0 || c->hidden <= 0 || c->max_seq <= 0 || (c->n_heads % c->n_kv_heads) != 0 ||
      (c->head_dim % 2) != 0)
    return NULL;
  oracle_model *m = (oracle_model *)calloc(1, sizeof *m);
  m->c = *c;
  m->act = mode_act(c->mode);
  m->i8 = mode_int8(c->mode);
  m->q_dim = c->n_heads * c->head_dim;
  m->kv_dim = c->n_kv_heads * c->head_dim;
  m->group = c->n_heads / c->n_kv_heads;
  size_t ne = (size_t)c->vocab * c->dim;
  if (m->act) {
    m->embed_r = (float *)malloc(sizeof(float) * ne);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < ne; i++) m->embed_r[i] = round_act(m->act, w->embed[i]);
    m->embed = m->embed_r;
    if (w->lm_head) {
      m->lm_head_r = (float *)malloc(sizeof(float) * ne);
#pragma omp parallel for schedule(static)
      for (size_t i = 0; i < ne; i++) m->lm_head_r[i] = round_act(m->act, w->lm_head[i]);
      m->lm_head = m->lm_head_r;
    } else {
      m->lm_head = m->embed_r;
    }
  } else {
    m->embed = w->embed;
    m->lm_head = w->lm_head ? w->lm_head : w->embed;
  }
  m->rms_final = w->rms_final;
  m->layers = (layer_t *)calloc((size_t)c->n_layers, sizeof(layer_t));
  for (int l = 0; l < c->n_layers; l++) {
    const oracle_layer_f32 *s = &w->layers[l];
    layer_t *d = &m->layers[l];
    mat_init(&d->wq, s->wq, m->q_dim, c->dim, m->act, m->i8);
    mat_init(&d->wk, s->wk, m->kv_dim, c->dim, m->act, m->i8);
    mat_init(&d->wv, s->wv, m->kv_dim, c->dim, m->act, m->i8);
    mat_init(&d->wo, s->wo, c->dim, m->q_dim, m->act, m->i8);
    mat_init(&d->w1, s->w1, c->hidden, c->dim, m->act, m->i8);
    mat_init(&d->w2, s->w2, c->dim, c->hidden, m->act, m->i8);
    mat_init(&d->w3, s->w3, c->hidden, c->dim, m->act, m->i8);
    d->rms_att = s->rms_att;
    d->rms_ffn = s->rms_ffn;
    d->q_norm = s->q_norm;
    d->k_norm = s->k_norm;
  }
  int half = c->head_dim / 2;
  m->rope_cos = (float *)malloc(sizeof(float) * (size_t)c->max_seq * half);
  m->rope_sin = (float *)malloc(sizeof(float) * (size_t)c->max_seq * half);
  oracle_rope_tables(c->max_seq, c->head_dim, c->rope_theta, m->rope_cos, m->rope_sin);
  return m;
}

void oracle_model_free(oracle_model *m) {
  if (!m) return;
  for (int l = 0; l < m->c.n_layers; l++) {
    layer_t *d = &m->layers[l];
    mat_free(&d->wq); mat_free(&d->wk); mat_free(&d->wv); mat_free(&d->wo);
    mat_free(&d->w1); mat_free(&d->w2); mat_free(&d->w3);
  }
  free(m->layers);
  free(m->embed_r);
  free(m->lm_head_r);
  free(m->rope_cos);
  free(m->rope_sin);
  free(m);
}

oracle_seq *oracle_seq_new(const oracle_model *m) {
  if (!m) return NULL;
  const oracle_config *c = &m->c;
  oracle_seq *s = (oracle_seq *)calloc(1, sizeof *s);
  s->m = m;
  size_t kv = (size_t)c->n_layers * c->max_seq * m->kv_dim;
  s->kcache = (float *)calloc(kv, sizeof(float));
  s->vcache = (float *)calloc(kv, sizeof(float));
  int wide = c->dim > m->q_dim ? c->dim : m->q_dim;
  if (c->hidden > wide) wide = c->hidden;
  s->x = (float *)calloc((size_t)c->dim, sizeof(float));
  s->xn = (float *)calloc((size_t)wide, sizeof(float));
  s->q = (float *)calloc((size_t)m->q_dim, sizeof(float));
  s->k = (float *)calloc((size_t)m->kv_dim, sizeof(float));
  s->v = (float *)calloc((size_t)m->kv_dim, sizeof(float));
  s->att = (float *)calloc((size_t)m->q_dim, sizeof(float));
  s->x2 = (float *)calloc((size_t)c->dim, sizeof(float));
  s->h1 = (float *)calloc((size_t)c->hidden, sizeof(float));
  s->h3 = (float *)calloc((size_t)c->hidden, sizeof(float));
  s->g = (float *)calloc((size_t)c->hidden, sizeof(float));
  s->y = (float *)calloc((size_t)wide, sizeof(float));
  s->logits = (float *)calloc((size_t)c->vocab, sizeof(float));
  s->qa = (int8_t *)calloc((size_t)wide, 1);
  return s;
}

void oracle_seq_free(oracle_seq *s) {
  if (!s) return;
  free(s->kcache); free(s->vcache); free(s->x); free(s->xn); free(s->q); free(s->k); free(s->v);
  free(s->att); free(s->x2); free(s->h1); free(s->h3); free(s->g); free(s->y); free(s->logits);
  free(s->qa);
  free(s);
}

/* ane/stories/infer.go:62-71 */
void oracle_seq_reset(oracle_seq *s) {
  if (!s) return;
  size_t kv = (size_t)s->m->c.n_layers * s->m->c.max_seq * s->m->kv_dim;
  memset(s->kcache, 0, kv * sizeof(float));
  memset(s->vcache, 0, kv * sizeof(float));
}

static uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

/* The sampling uniform of the CUDA path's documented generator: a per-stream key from the
 * seed, then SplitMix64 of key + counter, top 53 bits scaled to [0, 1). */
double oracle_uniform(uint64_t seed, uint64_t stream, uint64_t counter) {
  const uint64_t key = splitmix64(seed ^ splitmix64(stream * 0xD1B54A32D192ED03ull + 0x8CB92BA72F3D8DD7ull));
  return (double)(splitmix64(key + counter) >> 11) * (1.0 / 9007199254740992.0);
}

/* ane/stories/infer.go:347-371 sampleFromLogits with the uniform u given: temperature <= 1e-6
 * -> argmax; else f32 max, invT = float64(f32 1/temperature), total = sequential float64 sum
 * of exp((f64(l) - f64(mx)) * invT), target = u * total, first i whose running sum >= target,
 * else n - 1. */
int oracle_sample_from_logits(const float *logits, int n, float temperature, double u) {
  if (temperature <= 1e-6f) return oracle_argmax(logits, n);
  float mx = logits[0];
  for (int i = 1; i < n; i++)
    if (logits[i] > mx) mx = logits[i];
  const double inv_t = (double)(1.0f / temperature);
  double total = 0.0;
  for (int i = 0; i < n; i++) total += exp(((double)logits[i] - (double)mx) * inv_t);
  const double target = u * total;
  double acc = 0.0;
  for (int i = 0; i < n; i++) {
    acc += exp(((double)logits[i] - (double)mx) * inv_t);
    if (acc >= target) return i;
  }
  return n - 1;
}

void oracle_seq_fill_kv_synthetic(const oracle_model *m, oracle_seq *s, int n_pos, uint64_t seed) {
  const oracle_config *c = &m->c;
  if (n_pos > c->max_seq) n_pos = c->max_seq;
  for (int l = 0; l < c->n_layers; l++)
    for (int p = 0; p < n_pos; p++)
      for (int i = 0; i < m->kv_dim; i++) {
        size_t idx = ((size_t)l * c->max_seq + p) * m->kv_dim + i;
        uint64_t r = splitmix64(seed + idx);
        float u = (float)((double)(r >> 11) * (1.0 / 9007199254740992.0)) - 0.5f;
        s->kcache[idx] = round_act(m->act, u);
        s->vcache[idx] = round_act(m->act, 0.5f * u);
      }
}

/* ane/stories/infer.go:313-322 -- one serial f32 sum per output row (rows in parallel). */
static void matvec_f32(float *out, const float *mat, const float *in, int rows, int cols) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    const float *row = mat + (size_t)r * cols;
    float sum = 0.0f;
    if (g_matvec_reverse)
      for (int c = cols - 1; c >= 0; c--) sum += row[c] * in[c];
    else
      for (int c = 0; c < cols; c++) sum += row[c] * in[c];
    out[r] = sum;
  }
}

/* W8A8 linear: exact int32 dot of per-token-quantised input with the per-channel int8 row,
 * dequantised as (float)acc * s_act * s_w. */
static void matvec_i8(float *out, const mat_t *mt, const int8_t *qa, float sa) {
  int rows = mt->rows, cols = mt->cols;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    const int8_t *row = mt->q + (size_t)r * cols;
    int32_t acc = 0;
    for (int c = 0; c < cols; c++) acc += (int32_t)row[c] * (int32_t)qa[c];
    out[r] = oracle_dequant(acc, sa, mt->s[r]);
  }
}

/* Linear layer on an activation vector that is already normalised (f32):
 * F32 mode: matVec as the reference; fp16/bf16: round the input, matVec on rounded weights;
 * W8A8: quantise the input per token, int8 matVec. `in` is rounded in place. */
static void linear(oracle_seq *s, float *out, const mat_t *mt, float *in) {
  const oracle_model *m = s->m;
  if (m->i8) {
    float sa = quant_row(in, mt->cols, s->qa);
    matvec_i8(out, mt, s->qa, sa);
  } else {
    round_vec(m->act, in, mt->cols);
    matvec_f32(out, mt->fp, in, mt->rows, mt->cols);
  }
}

/* Two linears sharing the same (normalised) input, quantised/rounded once. */
static void linear2(oracle_seq *s, float *o1, const mat_t *m1, float *o2, const mat_t *m2, float *in) {
  const oracle_model *m = s->m;
  if (m->i8) {
    float sa = quant_row(in, m1->cols, s->qa);
    matvec_i8(o1, m1, s->qa, sa);
    matvec_i8(o2, m2, s->qa, sa);
  } else {
    round_vec(m->act, in, m1->cols);
    matvec_f32(o1, m1->fp, in, m1->rows, m1->cols);
    matvec_f32(o2, m2->fp, in, m2->rows, m2->cols);
  }
}

/* ane/stories/infer.go:247-265 generalised to n heads of width hd. */
static void apply_rope(const oracle_model *m, float *v, int nheads, int pos) {
  int hd = m->c.head_dim, half = hd / 2;
  const float *cs = m->rope_cos + (size_t)pos * half, *sn = m->rope_sin + (size_t)pos * half;
  for (int h = 0; h < nheads; h++) {
    float *b = v + (size_t)h * hd;
    for (int i = 0; i < half; i++) {
      float c = cs[i], s = sn[i];
      float a0 = b[2 * i], a1 = b[2 * i + 1];
      b[2 * i] = a0 * c - a1 * s;
      b[2 * i + 1] = a0 * s + a1 * c;
    }
  }
}

/* ane/stories/infer.go:267-299 with the GQA map of training/training_dynamic/io.h:434-455. */
static void attend(oracle_seq *s, int layer, int pos) {
  const oracle_model *m = s->m;
  const oracle_config *c = &m->c;
  int hd = c->head_dim;
  float inv_sqrt_hd = (float)(1.0 / sqrt((double)hd));
  const float *kc = s->kcache + (size_t)layer * c->max_seq * m->kv_dim;
  const float *vc = s->vcache + (size_t)layer * c->max_seq * m->kv_dim;
  int n = pos + 1;
#pragma omp parallel for schedule(static)
  for (int h = 0; h < c->n_heads; h++) {
    float *scores = (float *)malloc(sizeof(float) * (size_t)n);
    float *probs = (float *)malloc(sizeof(float) * (size_t)n);
    int kvh = h / m->group;
    const float *qh = s->q + (size_t)h * hd;
    for (int t = 0; t <= pos; t++) {
      const float *kt = kc + (size_t)t * m->kv_dim + (size_t)kvh * hd;
      float dot = 0.0f;
      for (int i = 0; i < hd; i++) dot += qh[i] * kt[i];
      scores[t] = dot * inv_sqrt_hd;
    }
    float *out = s->att + (size_t)h * hd;
    if (!m->act) {
      oracle_softmax_prefix(probs, scores, n);
      for (int i = 0; i < hd; i++) {
        float sum = 0.0f;
        for (int t = 0; t <= pos; t++) sum += probs[t] * vc[(size_t)t * m->kv_dim + (size_t)kvh * hd + i];
        out[i] = sum;
      }
    } else {
      /* Emulation: the CUDA kernel carries the softmax weights exp(s - max) at ~fp32
       * precision (a two-term split in the activation type) and divides by the f32 sum at
       * the end; q, K and V are already rounded to the activation type. */
      float mx = scores[0];
      for (int t = 1; t < n; t++)
        if (scores[t] > mx) mx = scores[t];
      double sum = 0.0;
      for (int t = 0; t < n; t++) {
        float e = (float)exp((double)(scores[t] - mx));
        probs[t] = e;
        sum += (double)e;
      }
      float inv = (float)(1.0 / sum);
      for (int i = 0; i < hd; i++) {
        float acc = 0.0f;
        if (g_attn_reverse)
          for (int t = pos; t >= 0; t--) acc += probs[t] * vc[(size_t)t * m->kv_dim + (size_t)kvh * hd + i];
        else
          for (int t = 0; t <= pos; t++) acc += probs[t] * vc[(size_t)t * m->kv_dim + (size_t)kvh * hd + i];
        out[i] = acc * inv;
      }
    }
    free(scores);
    free(probs);
  }
}

/* ane/stories/infer.go:204-245 (generalised; see oracle.h). */
int oracle_forward(const oracle_model *m, oracle_seq *s, int token, int pos, float *logits_out) {
  if (!m || !s) return ORACLE_EINVAL;
  const oracle_config *c = &m->c;
  if (token < 0 || token >= c->vocab) return ORACLE_ERANGE_TOKEN;
  if (pos < 0 || pos >= c->max_seq) return ORACLE_ERANGE_POS;
  int D = c->dim, F = c->hidden, hd = c->head_dim;

  memcpy(s->x, m->embed + (size_t)token * D, sizeof(float) * (size_t)D);
  for (int l = 0; l < c->n_layers; l++) {
    const layer_t *L = &m->layers[l];
    oracle_rmsnorm(s->xn, s->x, L->rms_att, D, c->norm_eps);
    if (m->i8) {
      float sa = quant_row(s->xn, D, s->qa);
      matvec_i8(s->q, &L->wq, s->qa, sa);
      matvec_i8(s->k, &L->wk, s->qa, sa);
      matvec_i8(s->v, &L->wv, s->qa, sa);
    } else {
      round_vec(m->act, s->xn, D);
      matvec_f32(s->q, L->wq.fp, s->xn, m->q_dim, D);
      matvec_f32(s->k, L->wk.fp, s->xn, m->kv_dim, D);
      matvec_f32(s->v, L->wv.fp, s->xn, m->kv_dim, D);
    }
    if (c->qk_norm) {
      for (int h = 0; h < c->n_heads; h++) oracle_rmsnorm(s->q + (size_t)h * hd, s->q + (size_t)h * hd, L->q_norm, hd, c->norm_eps);
      for (int h = 0; h < c->n_kv_heads; h++) oracle_rmsnorm(s->k + (size_t)h * hd, s->k + (size_t)h * hd, L->k_norm, hd, c->norm_eps);
    }
    apply_rope(m, s->q, c->n_heads, pos);
    apply_rope(m, s->k, c->n_kv_heads, pos);
    round_vec(m->act, s->q, m->q_dim);
    round_vec(m->act, s->k, m->kv_dim);
    round_vec(m->act, s->v, m->kv_dim);
    size_t base = ((size_t)l * c->max_seq + pos) * m->kv_dim;
    memcpy(s->kcache + base, s->k, sizeof(float) * (size_t)m->kv_dim);
    memcpy(s->vcache + base, s->v, sizeof(float) * (size_t)m->kv_dim);
    attend(s, l, pos);
    linear(s, s->x2, &L->wo, s->att);
    if (m->resid_scale != 0.0f) /* ane/storiesane/accel_other.go:60-64: base + scale*branch */
      for (int i = 0; i < D; i++) s->x2[i] = s->x[i] + m->resid_scale * s->x2[i];
    else
      for (int i = 0; i < D; i++) s->x2[i] += s->x[i];

    oracle_rmsnorm(s->xn, s->x2, L->rms_ffn, D, c->norm_eps);
    linear2(s, s->h1, &L->w1, s->h3, &L->w3, s->xn);
    if (m->silu_form) /* ane/storiesane/accel_other.go:66-71 */
      for (int i = 0; i < F; i++) {
        float sig = (float)(1.0 / (1.0 + exp(-(double)s->h1[i])));
        s->g[i] = (s->h1[i] * sig) * s->h3[i];
      }
    else
      for (int i = 0; i < F; i++) s->g[i] = oracle_silu(s->h1[i]) * s->h3[i];
    linear(s, s->y, &L->w2, s->g);
    if (m->resid_scale != 0.0f)
      for (int i = 0; i < D; i++) s->x[i] = s->x2[i] + m->resid_scale * s->y[i];
    else
      for (int i = 0; i < D; i++) s->x[i] = s->x2[i] + s->y[i];
  }
  oracle_rmsnorm(s->xn, s->x, m->rms_final, D, c->norm_eps);
  round_vec(m->act, s->xn, D);
  matvec_f32(s->logits, m->lm_head, s->xn, c->vocab, D);
  if (logits_out) memcpy(logits_out, s->logits, sizeof(float) * (size_t)c->vocab);
  return ORACLE_OK;
}

/* ane/stories/infer.go:136-202, greedy (temperature <= 1e-6). */
int oracle_decode(const oracle_model *m, oracle_seq *s, const int32_t *prompt, int n_prompt, int max_new,
                  int32_t *out_tokens, int32_t *n_tokens, int32_t *prompt_len, int32_t *stopped_on_eos) {
  if (!m || !s) return ORACLE_EINVAL;
  const oracle_config *c = &m->c;
  int max_seq = c->max_seq;
  if (max_new <= 0) max_new = 64;
  int32_t bos = BOS_TOKEN;
  if (n_prompt <= 0) { prompt = &bos; n_prompt = 1; }
  if (n_prompt > max_seq) { prompt += n_prompt - max_seq; n_prompt = max_seq; }
  for (int i = 0; i < n_prompt; i++)
    if (prompt[i] < 0 || prompt[i] >= c->vocab) return ORACLE_ERANGE_TOKEN;
  oracle_seq_reset(s);
  int n = 0;
  for (int i = 0; i < n_prompt; i++) out_tokens[n++] = prompt[i];
  for (int pos = 0; pos < n_prompt - 1; pos++) {
    int rc = oracle_forward(m, s, prompt[pos], pos, NULL);
    if (rc) return rc;
  }
  int eos = 0;
  for (int step = 0; step < max_new && n < max_seq; step++) {
    int pos = n - 1;
    int rc = oracle_forward(m, s, out_tokens[pos], pos, NULL);
    if (rc) return rc;
    int next = oracle_argmax(s->logits, c->vocab);
    out_tokens[n++] = next;
    if (next == EOS_TOKEN) { eos = 1; break; }
  }
  *n_tokens = n;
  *prompt_len = n_prompt;
  *stopped_on_eos = eos;
  return ORACLE_OK;
}

int oracle_teacher_forced(const oracle_model *m, oracle_seq *s, const int32_t *tokens, int n,
                          int32_t *argmax_out, float *logits_out) {
  if (!m || !s) return ORACLE_EINVAL;
  oracle_seq_reset(s);
  for (int i = 0; i < n; i++) {
    int rc = oracle_forward(m, s, tokens[i], i, logits_out ? logits_out + (size_t)i * m->c.vocab : NULL);
    if (rc) return rc;
    if (argmax_out) argmax_out[i] = oracle_argmax(s->logits, m->c.vocab);
  }
  return ORACLE_OK;
}
