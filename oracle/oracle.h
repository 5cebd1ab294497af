/*
 * oracle.h -- CPU restatement of the reference token loop (TEST INFRASTRUCTURE).
 *
 * This library is the checker for the CUDA token loop.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs load
 * it; the product library never links or calls it.
 *
 * What it restates (file:line in the reference project tmc/ane-training-experiments):
 *   ane/stories/infer.go:80-133   NewDecoder: RoPE tables (float64 pow/cos/sin -> f32),
 *                                 KV cache [layer][pos][kv_dim]
 *   ane/stories/infer.go:136-202  Decode: prompt prefill one token at a time, greedy loop,
 *                                 EOS (id 2) stop, maxSeq stop, BOS (id 1) default prompt
 *   ane/stories/infer.go:204-245  forwardOne: layer order and residual form
 *   ane/stories/infer.go:247-265  applyRoPE: interleaved (2i, 2i+1) pairs
 *   ane/stories/infer.go:267-299  storeKV / attend (f32 dot, * 1/sqrt(hd), softmaxPrefix, PV)
 *   ane/stories/infer.go:301-311  rmsNormVec: float64 sum of squares, f32 rrms, x*rrms*w
 *   ane/stories/infer.go:313-322  matVec: serial f32 sum per output row
 *   ane/stories/infer.go:324-326  silu via float64 exp
 *   ane/stories/infer.go:328-345  softmaxPrefix: f32 max, float64 exp/sum, f32 probs
 *   ane/stories/infer.go:347-371  sampleFromLogits (uniform given; Go's math/rand is not restated)
 *   ane/stories/infer.go:373-383  argmax: strict '>' (first maximum wins)
 *   ane/storiesane/engine.go:804-842, decode.go:83-94  storiesane full-window forward (residual
 *                                 scale, gate form) and the BOS left-padded decode window
 *   training/training_dynamic/io.h:434-455   GQA head map kv_head = q_head / (heads/kv_heads)
 *   bridge/ane_bridge.m:374-398   int8 quantiser: scale = maxabs/127 (0 -> 1), v = x/scale,
 *                                 clamp [-128,127], (int8)(v + (v>=0 ? 0.5 : -0.5))
 *
 * Generalisations beyond the Go decoder (which hard-codes Stories110M):
 *   kv_heads / head_dim / QK-norm (per-head RMSNorm of q and k before RoPE) / theta / eps /
 *   max_seq without the 256 clamp, and precision-emulation modes that round at exactly the
 *   points where the CUDA path rounds (fp16/bf16 weights, GEMM inputs, KV cache, q, the
 *   attention output, the SwiGLU output) and that quantise like the CUDA W8A8 path
 *   (per-output-channel weight scales, per-token activation scales, both with the bridge
 *   rule applied row-wise).  Softmax weights are not rounded (the CUDA kernel carries them
 *   as a two-term split with ~16 mantissa bits).
 *
 * PARITY UNPINNED: the reference publishes no golden tokens/logits for this path and its Go
 * code cannot be run in this environment (no Go toolchain, and the module's tmc/apple
 * dependency is replaced to a path that does not exist).  The building blocks are pinned
 * by the known-answer tests under tests/ that restate the reference's own unit tests and
 * hand-derived values; the end-to-end decoder is pinned only by self-consistency fixtures.
 */
#ifndef ORACLE_H
#define ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ORACLE_F32 = 0,        /* the reference arithmetic, unchanged                    */
  ORACLE_F16 = 1,        /* fp16 weights / GEMM inputs / KV, f32 accumulate         */
  ORACLE_BF16 = 2,       /* bf16 weights / GEMM inputs / KV, f32 accumulate         */
  ORACLE_W8A8_F16 = 3,   /* int8 layer weights + per-token int8 acts, fp16 rest     */
  ORACLE_W8A8_BF16 = 4,  /* int8 layer weights + per-token int8 acts, bf16 rest     */
};

typedef struct oracle_config {
  int32_t dim, hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab;
  int32_t max_seq;
  int32_t qk_norm;     /* 1: per-head RMSNorm on q and k before RoPE (Qwen3) */
  int32_t mode;        /* ORACLE_* */
  double norm_eps;     /* Go uses the float64 constant 1e-5 */
  double rope_theta;   /* Go uses 10000 */
} oracle_config;

typedef struct oracle_layer_f32 {
  const float *wq, *wk, *wv, *wo;   /* [q_dim,dim] [kv_dim,dim] [kv_dim,dim] [dim,q_dim] */
  const float *w1, *w2, *w3;        /* [hidden,dim] [dim,hidden] [hidden,dim]            */
  const float *rms_att, *rms_ffn;   /* [dim]                                              */
  const float *q_norm, *k_norm;     /* [head_dim] (only read when qk_norm)                */
} oracle_layer_f32;

typedef struct oracle_weights_f32 {
  const float *embed;      /* [vocab, dim] */
  const float *rms_final;  /* [dim] */
  const float *lm_head;    /* [vocab, dim] or NULL when tied to embed */
  const oracle_layer_f32 *layers;
} oracle_weights_f32;

typedef struct oracle_model oracle_model;
typedef struct oracle_seq oracle_seq;

/* Error codes (negative), mirroring the C-ABI's. */
#define ORACLE_OK 0
#define ORACLE_EINVAL -1
#define ORACLE_ERANGE_TOKEN -2
#define ORACLE_ERANGE_POS -3

oracle_model *oracle_model_new(const oracle_config *cfg, const oracle_weights_f32 *w);
/* 1: the storiesane CPU forward's arithmetic (ane/storiesane/engine.go:804-842): residual
 * x + a*branch with a = float32(1/sqrt(2*layers)) (residual.go:9, accel_other.go:60-64) and
 * the gate (h1 * f32(1/(1+exp(-h1)))) * h3 (accel_other.go:66-71); 0: stories.Decoder's. */
void oracle_model_set_storiesane(oracle_model *m, int on);
/* 1: the CUDA path's order of operations, restated step for step so that the oracle's
 * results equal the GPU's bit for bit (emulation modes only; the reference's arithmetic is
 * the default):
 *   - RMSNorm sums of squares in the row kernel's lane order, QK-norm per 32-column chunk;
 *   - every 16-bit matVec (layers and lm_head) and every attention score / PV product as the
 *     tensor cores form them (oracle_mma16), in 16-term instructions in the kernels' order;
 *   - exp as exp2_det, the SwiGLU gate h1 / (1 + e) (or storiesane's h1 * (1 / (1 + e)));
 *   - attention of positions below oracle_seq_set_prefill's count in the prefill kernel's
 *     order (64-position tiles, lazy reference max), later positions in the decode kernel's
 *     (32-page segments, 4 warps, fixed fold order). */
void oracle_model_set_gpu_order(oracle_model *m, int on);
/* GPU order: whether a decode step's 16-bit residual projections (Wo, W2) split K over
 * clusters (the library's LLM_OPT_DECODE_SPLITK, default on), and the split of such a
 * projection: out channels n, input k, widest channel tile bnmax (256). */
void oracle_model_set_decode_splitk(oracle_model *m, int on);
int oracle_decode_splits(int in8, int n, int k, int bnmax);
/* C[m][n] of oracle_gemm_mma with K split into S ranges of 64-element slices (one MMA chain
 * each, partials added in range order, each addition rounded to nearest). */
void oracle_gemm_mma_splitk(const float *A, const float *B, int M, int N, int K, int act, int S, float *Cout);
void oracle_model_free(oracle_model *m);
oracle_seq *oracle_seq_new(const oracle_model *m);
void oracle_seq_free(oracle_seq *s);
void oracle_seq_reset(oracle_seq *s);
/* GPU order: positions [0, n_prefill) were computed by the prefill kernels (a prompt). */
void oracle_seq_set_prefill(oracle_seq *s, int n_prefill);
/* Forward passes at positions below `pos` skip the classifier (their logits read as zeros):
 * for long teacher-forced prompts whose logits are not compared.  Default 0. */
void oracle_seq_set_logits_from(oracle_seq *s, int pos);
/* The seeded N(0, stddev) weight generator of the synthetic models (SplitMix64 -> Box-Muller in
 * double, one rounding to f32; element i depends on (seed, stream, i) only) and its stream ids
 * (layer l, kind 0..6 = Wq Wk Wv Wo W1 W2 W3; 7 embedding; 8 untied classifier). */
void oracle_synth_normal(float *dst, uint64_t n, uint64_t seed, uint64_t stream, double stddev, double scale);
uint64_t oracle_synth_stream(int layer, int kind);
/* Fill the KV cache positions [0, n_pos) with seeded values (for timing samples only). */
void oracle_seq_fill_kv_synthetic(const oracle_model *m, oracle_seq *s, int n_pos, uint64_t seed);
/* forwardOne: returns ORACLE_OK or an error; logits_out may be NULL. */
int oracle_forward(const oracle_model *m, oracle_seq *s, int token, int pos, float *logits_out);
/* Decode (greedy; temperature <= 1e-6 branch of sampleFromLogits).  out_tokens receives
 * prompt + generated tokens (capacity max_seq).  Returns ORACLE_OK or an error. */
int oracle_decode(const oracle_model *m, oracle_seq *s, const int32_t *prompt, int n_prompt,
                  int max_new, int32_t *out_tokens, int32_t *n_tokens, int32_t *prompt_len,
                  int32_t *stopped_on_eos);
/* Teacher-forced pass: feed tokens[0..n) at positions 0..n-1; argmax_out[i] = argmax after
 * token i; logits_out (optional) gets [n, vocab]. */
int oracle_teacher_forced(const oracle_model *m, oracle_seq *s, const int32_t *tokens, int n,
                          int32_t *argmax_out, float *logits_out);

/* ---- building blocks (known-answer and bit-exact checks) ---- */
int oracle_argmax(const float *v, int n);
/* ane/stories/infer.go:347-371 with the uniform given (Go draws it from math/rand). */
int oracle_sample_from_logits(const float *logits, int n, float temperature, double u);
/* The CUDA path's counter-based uniform in [0, 1) (stream = sampling stream base + slot). */
double oracle_uniform(uint64_t seed, uint64_t stream, uint64_t counter);
void oracle_rmsnorm(float *out, const float *x, const float *w, int n, double eps);
void oracle_rope_tables(int max_pos, int head_dim, double theta, float *cos_out, float *sin_out);
void oracle_softmax_prefix(float *dst, const float *src, int n);
float oracle_silu(float x);
float oracle_round_f16(float x);
float oracle_round_bf16(float x);
/* Bridge quantiser applied per row (rows x cols); scales[rows]. */
void oracle_quant_rows(const float *x, int rows, int cols, int8_t *q, float *scales);
/* RMSNorm then per-row quantisation, with the float64 sum of squares taken in the order
 * the CUDA row kernel documents (per-thread float4 groups, per-warp xor butterfly, warp
 * totals in order; see sumsq_lane_order in oracle.c). */
void oracle_norm_quant_rows_lane_order(const float *x, const float *w, int rows, int cols,
                                       double eps, int8_t *q, float *scales);
/* Same lane-ordered RMSNorm without quantisation, output rounded per mode (F16/BF16/none). */
void oracle_norm_rows_lane_order(const float *x, const float *w, int rows, int cols,
                                 double eps, int round_mode, float *out);
/* 2^x from round-to-nearest f32 steps (the CUDA path's exp2_det; 0 below -126). */
float oracle_exp2_det(float x);
/* One tensor-core MMA step of n <= 16 products with fp16 (act 1) or bf16 (act 2) operands and
 * an f32 accumulator c, as measured on B200 (mma.sync.m16n8k16 and tcgen05.mma kind::f16 give
 * the same bits): exact products; each term (c included) truncated toward zero to a multiple of
 * 2^(E - 26), E the largest alignment exponent (e(a) + e(b) + 1 for a product, e(c) + 1 for
 * c, e = exponent of the leading bit); the exact sum rounded toward zero to f32. */
float oracle_mma16(float c, const float *a, const float *b, int n, int act);
/* C[m][n] = the MMA chain (oracle_mma16 over 16-term k slices in order, the first without
 * accumulator) of A[m][:] and B[n][:], K a multiple of 16: a 16-bit GEMM without split-K. */
void oracle_gemm_mma(const float *A, const float *B, int M, int N, int K, int act, float *C);
/* ane/stories/cpu.go:41-72 EmbedLookup (channel-first [dim][seq]; out-of-range tokens zero
 * their column). */
void oracle_embed_lookup_cf(float *out, const float *embed, int vocab, const int32_t *tokens, int dim, int seq);
/* Exact int8 GEMM: C[m][n] = sum_k A[m][k]*B[n][k]. */
void oracle_gemm_i8(const int8_t *A, const int8_t *B, int M, int N, int K, int32_t *C);
/* Dequantise an int32 accumulator the way the CUDA epilogue does: (float)acc*sa*sw. */
float oracle_dequant(int32_t acc, float sa, float sw);

/* Test-only: 1 = sum the attention PV products in reverse position order (emulation modes). */
void oracle_set_attn_reverse(int on);
/* Test-only: 1 = sum every f32 matVec (fp32 / fp16 / bf16 modes) in reverse column order. */
void oracle_set_matvec_reverse(int on);
/* Thread count used by row-parallel loops (OpenMP); 0 = library default. */
void oracle_set_threads(int n);
int oracle_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
