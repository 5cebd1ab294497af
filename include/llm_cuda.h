/*
 * llm_cuda.h -- C ABI of the B200 token loop (prefill + greedy decode) for the Llama-style
 * models of tmc/ane-training-experiments (Stories110M MHA, Qwen3-0.6B GQA).
 *
 * This is the boundary a cgo shim binds.  Plain C types only: opaque
 * handles, int status codes, host pointers and sizes.  The context owns all device memory;
 * the caller owns every host buffer it passes.  Status: 0 = LLM_OK, negative = error, with
 * the message available from llm_last_error() (precedent: bridge/stories_trainer_bridge.h:32-36,
 * bridge/ane_bridge.h:25-27).  A context is not thread-safe; serialise calls per context
 * (precedent: the per-kernel mutex of ane/linear/executor.go:44-50).
 *
 * There is no CPU fallback: every compute entry point runs CUDA kernels on the context's
 * device and fails with LLM_ERR_CUDA when that is impossible.
 */
#ifndef LLM_CUDA_H
#define LLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
#define LLM_OK 0
#define LLM_ERR_INVALID -1      /* bad argument / configuration                        */
#define LLM_ERR_TOKEN_RANGE -2  /* "token out of range: %d"    (ane/stories/infer.go:205-207) */
#define LLM_ERR_POS_RANGE -3    /* "position out of range: %d" (ane/stories/infer.go:208-210) */
#define LLM_ERR_CUDA -4         /* CUDA runtime failure                                */
#define LLM_ERR_OOM -5          /* device or page-pool memory exhausted                */
#define LLM_ERR_STATE -6        /* call order (weights / KV cache not set up)          */
#define LLM_ERR_UNSUPPORTED -7  /* a mode this build does not implement                */
#define LLM_ERR_DEVICE -8       /* a kernel reported an error (bounded wait expired, bad page) */

/* ---------------------------------------------------------------- configuration */
/* Arithmetic of the CUDA path. */
#define LLM_DTYPE_F16 1       /* fp16 weights/activations/KV, fp32 accumulate          */
#define LLM_DTYPE_BF16 2      /* bf16 weights/activations/KV, fp32 accumulate          */
#define LLM_DTYPE_W8A8_F16 3  /* int8 layer weights (per-output-channel scales) and
                                 per-token int8 activations, int32 accumulate; fp16
                                 embeddings/lm_head/KV                                 */
#define LLM_DTYPE_W8A8_BF16 4 /* as above with bf16 embeddings/lm_head/KV              */

/* Runtime model description; replaces the compile-time constants of
 * ane/stories/config.go:3-18 and training/training_dynamic/models/qwen3_06b.h:6-16. */
typedef struct llm_model_config {
  int32_t dim;         /* model width D                                           */
  int32_t hidden;      /* SwiGLU width F                                          */
  int32_t n_layers;
  int32_t n_heads;     /* query heads                                             */
  int32_t n_kv_heads;  /* key/value heads (GQA when < n_heads)                    */
  int32_t head_dim;    /* 64 or 128                                               */
  int32_t vocab;
  int32_t max_seq;     /* RoPE table length = largest position + 1                */
  int32_t qk_norm;     /* 1: per-head RMSNorm of q and k before RoPE (Qwen3)      */
  int32_t tied_embed;  /* 1: lm_head = embedding (ane/stories/infer.go:243)       */
  double norm_eps;     /* RMSNorm epsilon (Go: float64 1e-5, infer.go:307)        */
  double rope_theta;   /* RoPE base (Go: 10000, infer.go:102)                     */
} llm_model_config;

/* fp32 host weights in the reference's row-major [out, in] layout
 * (ane/stories/weights.go:13-23: LayerWeights / ModelWeights). */
typedef struct llm_layer_weights_f32 {
  const float *wq, *wk, *wv, *wo, *w1, *w2, *w3;
  const float *rms_att, *rms_ffn;
  const float *q_norm, *k_norm; /* [head_dim], read only when qk_norm */
} llm_layer_weights_f32;

typedef struct llm_model_weights_f32 {
  const float *embed;     /* [vocab, dim] */
  const float *rms_final; /* [dim] */
  const float *lm_head;   /* [vocab, dim] or NULL when tied */
  const llm_layer_weights_f32 *layers; /* n_layers entries */
} llm_model_weights_f32;

typedef struct llm_ctx llm_ctx;

/* ---------------------------------------------------------------- errors */
/* Copies the calling thread's last error message (NUL-terminated, truncated to n).
 * Returns the full message length.  Replaces ane_bridge's last-error accessor. */
int llm_last_error(char *buf, size_t n);

/* ---------------------------------------------------------------- context / weights */
/* Create a context on CUDA device `device`.  Replaces model.Compile
 * (ane/model/model_darwin.go:138-171) and stories.NewDecoder's setup
 * (ane/stories/infer.go:80-133: RoPE tables). */
int llm_ctx_create(const llm_model_config *cfg, int dtype, int device, llm_ctx **out);
/* Release every device resource.  Replaces Kernel.Close (ane/model/model_darwin.go:542-556). */
int llm_ctx_destroy(llm_ctx *ctx);

/* Upload fp32 host weights; conversion (rounding to fp16/bf16, or the int8 quantiser of
 * bridge/ane_bridge.m:374-398 per output row) runs on the device.  Replaces the weight
 * blob staging of model.CompileOptions.WeightBlob (ane/model/model_other.go:13-24). */
int llm_load_weights_f32(llm_ctx *ctx, const llm_model_weights_f32 *w);

/* Weight file formats of llm_load_weights_file. */
#define LLM_WEIGHTS_LLAMA2C 1    /* llama2.c .bin: ane/stories/weights.go:49-122 (LoadPretrained)     */
#define LLM_WEIGHTS_CHECKPOINT 2 /* training checkpoint v2/v3: ane/stories/ckpt.go:237-447
                                    (LoadCheckpoint with no optimizer state)                      */

/* Stream the weights of a file to the device tensor by tensor (one matrix in host memory at a
 * time; rounding / int8 quantisation on the device as llm_load_weights_f32).  The header must
 * match the context's configuration; errors use the reference's texts ("config mismatch: got
 * dim=%d hidden=%d layers=%d", "bad checkpoint header magic=%x version=%d", "checkpoint config
 * mismatch", "read <tensor>: unexpected EOF").  Both formats use the embedding as the
 * classifier, as ane/stories/infer.go:243 does, so the configuration must be tied and without
 * QK-norm.  Replaces stories.LoadPretrained / stories.LoadCheckpoint + NewDecoder's copy. */
int llm_load_weights_file(llm_ctx *ctx, const char *path, int format);

/* Seeded synthetic weights, generated on the host by llm_synth_normal (streams below):
 * matrices N(0, 0.02); Wo and W2 additionally x out_proj_scale (Stories: 1/sqrt(2*12));
 * RMSNorm and QK-norm weights 1.  Stands in for stories.RandomInit (ane/stories/weights.go:124-153),
 * whose Go math/rand stream cannot be reproduced here. */
int llm_load_weights_synthetic(llm_ctx *ctx, uint64_t seed, float out_proj_scale);

/* Counter-based N(0, stddev) generator: element i of stream `stream` is a function of
 * (seed, stream, i) only (SplitMix64 -> Box-Muller in double, one rounding to f32).
 * value = (float)(stddev * scale * z).  Multithreaded, deterministic. */
void llm_synth_normal(float *dst, uint64_t n, uint64_t seed, uint64_t stream, double stddev, double scale);
/* Stream id of each synthetic tensor: kind 0..6 = wq,wk,wv,wo,w1,w2,w3 of `layer`,
 * kind 7 = embed (layer ignored), kind 8 = untied lm_head (layer ignored). */
uint64_t llm_synth_stream(int layer, int kind);

/* ---------------------------------------------------------------- paged KV cache */
/* Allocate the page pool for `max_seqs` sequence slots of up to `max_pos` positions in
 * pages of `page_tokens` (must be 16) positions.  Replaces the [layer][pos][dim] cache of
 * stories.NewDecoder (ane/stories/infer.go:113-114).  Also sizes activation buffers. */
int llm_kv_alloc(llm_ctx *ctx, int max_seqs, int max_pos, int page_tokens);
/* Return a sequence slot's pages to the pool.  Replaces Decoder.ResetCache
 * (ane/stories/infer.go:62-71) for one slot. */
int llm_seq_release(llm_ctx *ctx, int seq);

/* ---------------------------------------------------------------- token loop */
/* Prefill: for each of `nseq` sequences, run its `lens[i]` prompt tokens (concatenated in
 * `tokens`) at positions start_pos[i].. (start_pos NULL = 0) and return the greedy next
 * token after the last one.  logits (optional) receives [nseq, vocab] for that position.
 * Replaces the one-token-at-a-time prompt loop of Decoder.Decode (ane/stories/infer.go:171-175). */
int llm_prefill(llm_ctx *ctx, const int32_t *seq_ids, const int32_t *tokens, const int32_t *lens,
                const int32_t *start_pos, int nseq, int32_t *next_tokens, float *logits);

/* One decode step for n sequences: token tokens[i] at position positions[i] of slot
 * seq_ids[i]; writes the greedy next token (first maximum wins, infer.go:373-383) and,
 * optionally, logits [n, vocab].  Host buffers; host<->device copies are inside the call.
 * Replaces Decoder.forwardOne + sampleFromLogits at temperature 0 (infer.go:204-245,347-350)
 * and Decoder.EvalNextLogits (infer.go:62-77). */
int llm_decode_step(llm_ctx *ctx, const int32_t *seq_ids, const int32_t *tokens, const int32_t *positions,
                    int n, int32_t *next_tokens, float *logits);

/* Device-resident greedy loop (no per-token host synchronisation): begin copies the
 * initial tokens/positions and reserves pages for max_steps; steps enqueues `steps`
 * decode steps on the context stream (each feeds its tokens to the next); end waits and
 * copies out_tokens [steps_done, n].  llm_generate = begin + steps + end. */
int llm_generate_begin(llm_ctx *ctx, const int32_t *seq_ids, const int32_t *tokens, const int32_t *positions,
                       int n, int max_steps);
int llm_generate_steps(llm_ctx *ctx, int steps);
int llm_generate_end(llm_ctx *ctx, int32_t *out_tokens, int32_t *steps_done);
int llm_generate(llm_ctx *ctx, const int32_t *seq_ids, const int32_t *tokens, const int32_t *positions, int n,
                 int steps, int32_t *out_tokens);

/* ---------------------------------------------------------------- stories.Decoder mirror */
/* Greedy Decode of one sequence slot with the reference's host rules (ane/stories/infer.go:136-202):
 * empty prompt -> [BOS=1]; prompt longer than max_seq keeps its last max_seq tokens;
 * prompt tokens range-checked ("prompt token[%d]=%d out of range"); stop at max_new
 * (<= 0 -> 64), at max_seq, or after EOS=2.  temperature > 1e-6 samples (llm_set_sampling's
 * generator state, this call's temperature); otherwise greedy.
 * out_tokens needs max_seq entries; it receives prompt + generated tokens. */
int llm_stories_decode(llm_ctx *ctx, int seq, const int32_t *prompt, int n_prompt, int max_new,
                       float temperature, int32_t *out_tokens, int32_t *n_tokens, int32_t *prompt_len,
                       int32_t *stopped_on_eos);
/* The batched form: nseq independent slots 0..nseq-1, prompts concatenated; out_tokens is
 * [nseq, max_seq]; per-sequence n_tokens / prompt_len / stopped_on_eos. */
int llm_stories_decode_batch(llm_ctx *ctx, const int32_t *prompts, const int32_t *prompt_lens, int nseq,
                             int max_new, float temperature, int32_t *out_tokens, int32_t *n_tokens,
                             int32_t *prompt_len, int32_t *stopped_on_eos);

/* ---------------------------------------------------------------- full-window evaluation */
/* Layer arithmetic of llm_eval_window. */
#define LLM_ARITH_STORIES 0     /* stories.Decoder: x + branch, silu(h1) = h1 / (1 + exp(-h1))    */
#define LLM_ARITH_STORIESANE 1  /* storiesane CPU forward (ane/storiesane/engine.go:804-842):
                                   x + a * branch with a = float32(1/sqrt(2 * layers))
                                   (residual.go:9), gate = (h1 * sigmoid(h1)) * h3
                                   (accel_other.go:66-71)                                      */
/* One full window of `seq` tokens at positions 0..seq-1 from an empty cache in sequence slot
 * `slot` (released before and after): every position's logits, written channel-first as
 * logits_cf[vocab][seq] when non-NULL (the layout of storiesane.Engine.EvalLogits,
 * engine.go:363-376), and the next token after the last position in *next_token (greedy, or
 * sampled per llm_set_sampling from the slot's stream).  seq <= the KV cache's max_pos.  A
 * token outside [0, vocab) gives its position a zero embedding column (EmbedLookup,
 * ane/stories/cpu.go:41-72).  Replaces Engine.evalLogitsInto (engine.go:734-747) / evalLogitsCPUInto (:804-842); the
 * windowed Engine.Decode (decode.go:18-94) calls it once per generated token. */
int llm_eval_window(llm_ctx *ctx, int slot, const int32_t *tokens, int seq, int arithmetic,
                    int32_t *next_token, float *logits_cf);

/* ---------------------------------------------------------------- temperature sampling */
/* Sample the next tokens with `temperature` (> 1e-6; <= 1e-6 or negative = greedy argmax) as
 * sampleFromLogits does (ane/stories/infer.go:347-371: f32 max, invT = float64(1/T), f64
 * exp-sum inverse CDF, first index whose running sum reaches u * total, else vocab - 1) for
 * every following prefill / decode step / generate step, until changed.  u comes from a
 * counter-based generator (llm_sample_uniform) of `seed`, the row's sequence slot and that
 * slot's draw count, which each sample advances on the device; reset_draws != 0 zeroes every
 * slot's count (infer.go:150-152 reseeding).  Go's math/rand stream of the reference is not
 * reproduced (parity of the uniforms is unpinned; the sampler given the same u and logits is
 * checked against the oracle).  llm_stories_decode[_batch] take their temperature per call. */
int llm_set_sampling(llm_ctx *ctx, float temperature, uint64_t seed, int reset_draws);
/* The generator: u in [0, 1) for (seed, slot, counter); SplitMix64 of a per-slot key plus the
 * counter, top 53 bits. */
double llm_sample_uniform(uint64_t seed, int32_t slot, uint64_t counter);
/* Failure-path test hook: a kernel waits on an mbarrier that nothing completes, gives up after
 * `polls` polls and records the timeout like every bounded wait of the token loop; the call
 * returns LLM_ERR_DEVICE ("bounded wait expired") and the device stays usable. */
int llm_debug_wait_timeout(int device, uint32_t polls);
/* Test hook: the device sampler on host logits [rows, vocab] with explicit uniforms u[rows]. */
int llm_debug_sample(int device, const float *logits, int rows, int vocab, float temperature,
                     const double *u, int32_t *out);

/* ---------------------------------------------------------------- execution options */
#define LLM_OPT_CUDA_GRAPHS 1  /* replay each decode step as a captured CUDA graph (default 1)   */
#define LLM_OPT_TCGEN05_GEMM 2 /* tcgen05 projections (default 1); 0 = warp-level mma.sync ones   */
#define LLM_OPT_PDL 3          /* programmatic dependent launch between the kernels of single-stream
                                  steps and prefill chunks (default 1)                           */
#define LLM_OPT_OVERLAP 4      /* decode batches of >= 64 sequences run as micro-batches (of >= 32
                                  sequences, at most LLM_OPT_MICRO_BATCHES) on their own streams
                                  whose attention launches form a chain, overlapping one
                                  micro-batch's projections with the others' attention:
                                  0 never, 1 when the step's K/V streaming time covers the host's
                                  eager launches (default; see llm_step_parts), 2 always         */
#define LLM_OPT_OVERLAP_RING_KB 5 /* shared memory (KB) of a projection's stage ring in overlap
                                     mode, so it fits beside two attention CTAs (default 64)   */
#define LLM_OPT_ATTN_SPLITS 6  /* decode attention splits per sequence; 0 = chosen per batch (default) */
#define LLM_OPT_MICRO_BATCHES 8 /* most micro-batches of the overlapped schedule, 2..4 (default 4)  */
#define LLM_OPT_OVERLAP_GRAPHS 9 /* capture overlapped steps in CUDA graphs (default 0: eager launches,
                                    measured faster for this schedule)                          */
#define LLM_OPT_CHAIN_PDL 10    /* overlap mode: programmatic dependent launch between the kernels of a
                                    micro-batch's projection chain (attention excluded)        */
#define LLM_OPT_PREFILL_TILES 11 /* prefill attention by query tiles of 128/group positions (default 1);
                                     0 = the decode kernel's blocks of 8/group positions       */
#define LLM_OPT_PREFILL_RING_KB 13 /* stage ring (KB) of prefill-sized per-tile tcgen05 GEMMs (those
                                      the persistent kernel does not take), so two CTAs share an
                                      SM (default 64; 0 = the full ring)                          */
#define LLM_OPT_PREFILL_BN 14   /* channel tile of those per-tile GEMMs (64, 128, 256; default 128;
                                   0 = the widest)                                            */
#define LLM_OPT_PREFILL_TC 15   /* prefill query tiles on tcgen05 tensor cores (TMEM accumulators);
                                   0 = the mma.sync tile kernel (default 1)                   */
#define LLM_OPT_PREFILL_PERSIST 16  /* projections of >= 1024-row chunks on the persistent tcgen05
                                       kernel (double-buffered TMEM accumulators; default 1) */
#define LLM_OPT_DECODE_SPLITK 17 /* fp16 / bf16 models: a decode step's residual projections (Wo,
                                    W2) split K over a cluster of 2-4 CTAs whose partial tiles
                                    are summed in rank order through distributed shared memory
                                    (default 1; the split per projection is fixed by its shape,
                                    so results do not depend on the batch; the rounding differs
                                    from 0; int8 models never split) */
#define LLM_OPT_ATTN_CHAIN 7   /* overlap mode: a micro-batch's attention launch starts once every CTA of
                                  the other's has started (1, default) or once it completed (0)  */
/* Set an execution option (0/1 switches; sizes and counts where noted).  Results do not depend
 * on the options beyond fp32 summation order; cached graphs are dropped when an option
 * changes.  No counterpart in the
 * reference (its ANE runtime has no such switches). */
int llm_set_option(llm_ctx *ctx, int option, int value);

/* ---------------------------------------------------------------- introspection / timing */
/* The context's CUDA stream (cudaStream_t) so callers can record events on it. */
int llm_ctx_stream(llm_ctx *ctx, void **stream);
int llm_synchronize(llm_ctx *ctx);
/* Number of kernel launches one decode step of n sequences makes (for the contexts of the
 * last llm_decode_step / llm_generate_begin). */
int llm_step_kernel_count(llm_ctx *ctx, int n, int *count);
/* Micro-batches such a step runs as (1 = the single-stream, graph-replayed schedule).  The
 * overlapped schedule is chosen when the step's K/V bytes take the device longer to stream
 * than the host needs to enqueue the extra launches (it launches eagerly). */
int llm_step_parts(llm_ctx *ctx, int n, int *parts);
/* Device bytes held by the context (weights, KV pool, buffers, workspace). */
int llm_memory_bytes(llm_ctx *ctx, uint64_t *weights, uint64_t *kv_pool, uint64_t *other);
/* Time `iters` back-to-back launches of the attention kernel of every layer for the
 * current generate batch at the positions of its last executed step (at least one
 * llm_generate_steps step must have run) with CUDA events on the context stream; returns
 * the mean duration of one launch in microseconds and the algorithmic bytes one launch
 * reads and writes.  The generate state is left as it was. */
int llm_time_attention(llm_ctx *ctx, int iters, double *us_per_launch, double *bytes_per_launch);

/* Run `iters` decode steps of the current generate batch eagerly with a CUDA event after
 * every launch (tokens and positions are not advanced; the next step must still be within
 * the steps reserved by llm_generate_begin, since it writes K/V there) and write a per-kernel table
 * (count per step, us per launch, us per step, share) into report.  step_us receives the
 * eager step time (launch gaps included). */
int llm_profile_step(llm_ctx *ctx, int iters, char *report, size_t report_len, double *step_us);

/* Launch timeline of the next decode step of the current generate batch, run eagerly in the
 * current schedule (overlapped micro-batches included; tokens and positions are not advanced,
 * the step must be within the reserved ones): one report line per launch with its first CTA
 * start, the spread of CTA start times, the last CTA end (microseconds from the step's first
 * CTA, device globaltimer) and its CTA count.  step_us receives first start to last end. */
int llm_trace_step(llm_ctx *ctx, char *report, size_t report_len, double *step_us);
/* Record the launch timeline of every forward pass enqueued between llm_trace_begin and
 * llm_trace_end (prefill chunks, decode steps, window evaluations; at most 1024 launches),
 * then report it as llm_trace_step does.  While recording, decode steps launch eagerly (no
 * CUDA graph replay), so every launch carries its record. */
int llm_trace_begin(llm_ctx *ctx);
int llm_trace_end(llm_ctx *ctx, char *report, size_t report_len, double *span_us);

/* ---------------------------------------------------------------- linear kernels */
/* A 1x1 convolution y = W x on channel-first fp32 tensors, the unit the reference compiles and
 * evaluates per layer (model.Compile / Kernel.WriteInputF32 / EvalWithStats / ReadOutputF32,
 * ane/model/model_darwin.go:138-414; forward.ConvEval, ane/forward/conv.go:11-48), run as one
 * tcgen05 GEMM with the token loop's arithmetic: fp16 / bf16 round the weights and inputs and
 * accumulate in f32; W8A8 quantises each weight row and each input column (token) with the
 * bridge rule and accumulates in int32, y = (acc * s_x) * s_w. */
typedef struct llm_linear llm_linear;
/* Weights w [out_dim][in_dim] fp32 (row-major, the reference's layout), converted on `device`;
 * out_dim a multiple of 16, in_dim of 128. */
int llm_linear_create(int device, int dtype, const float *w, int out_dim, int in_dim, llm_linear **out);
/* x_cf [in_dim][s] -> y_cf [out_dim][s] (host buffers); hw_ns (optional) receives the device
 * time of the evaluation (EvalStats.HWExecutionNS). */
int llm_linear_eval_cf(llm_linear *k, const float *x_cf, int s, float *y_cf, uint64_t *hw_ns);
int llm_linear_destroy(llm_linear *k);

/* ---------------------------------------------------------------- multi-GPU jobs */
/* Sequences are independent (ane/stories/infer.go:136-245), so a multi-GPU job splits its
 * n_total sequences across ranks (one process per GPU) in contiguous blocks and gathers the
 * generated token ids once at the end; nothing crosses ranks while tokens are generated.
 * No counterpart in the reference (it decodes one sequence in one process). */
/* Rank `rank`'s block of an n_total-sequence job: [start, start + count); the first
 * n_total % nranks ranks hold one sequence more. */
int llm_shard_range(int n_total, int nranks, int rank, int *start, int *count);
typedef struct llm_comm llm_comm;
#define LLM_COMM_ID_BYTES 128
/* A new communicator id (on one rank; the host hands the bytes to every rank).  NCCL is
 * loaded on first use (LLM_ERR_UNSUPPORTED without it). */
int llm_comm_unique_id(unsigned char *id, size_t id_bytes);
/* Join communicator `id` as `rank` of `nranks` on CUDA device `device`.  Every wait of the
 * communicator is bounded by timeout_s seconds (<= 0: 60): a rank that never joins or never
 * takes part in a gather makes the others fail with LLM_ERR_DEVICE instead of hanging. */
int llm_comm_create(const unsigned char *id, size_t id_bytes, int nranks, int rank, int device, double timeout_s,
                    llm_comm **out);
int llm_comm_destroy(llm_comm *comm);
/* The job's one collective: every rank passes its [steps][n_local] host block of token ids
 * (n_local = its llm_shard_range count) and receives [steps][n_total] in global sequence order
 * (an all-gather over NVLink / NVSwitch; every rank must call it). */
int llm_gather_tokens(llm_comm *comm, const int32_t *tokens, int steps, int n_local, int n_total, int32_t *out);
/* Device time (CUDA events on the communicator's stream) of the last completed gather: the
 * copy of the block to the device and the all-gather. */
int llm_comm_last_gather_ms(llm_comm *comm, double *ms);

/* ---------------------------------------------------------------- allocation-free entry point */
/* No counterpart in the reference.  Split-K int8 GEMM C[M,N] = A[M,K] . B[N,K]^T with int32
 * output that allocates nothing: for callers that cannot allocate device memory while they
 * run (a server whose KV page pool already holds the GPU's memory, a decode loop that must not
 * take cudaFree's device-wide synchronisation mid-step, an FFI host that owns the memory
 * policy).  A, B and C are caller-owned DEVICE pointers; the work is enqueued on `stream`
 * (NULL = default stream) and the call returns without waiting.  A and B must be 16-byte and C
 * 4-byte aligned (LLM_ERR_INVALID otherwise).  The split partials and tile
 * counters live in one fixed device array of 4 MiB + 1024 counters inside the library; a
 * shape/split combination needing more is rejected with LLM_ERR_INVALID.  The first call on a
 * device resolves that array's device address and sets kernel attributes, so make it before
 * any stream capture.  Every call shares the array: calls whose executions overlap on the GPU
 * (other streams or threads) race. */
int llm_gemm_i8_splitk_noalloc(int device, const int8_t *A, const int8_t *B, int M, int N, int K, int splits,
                               int32_t *C, void *stream);

/* ---------------------------------------------------------------- bit-exact debug hooks */
/* RMSNorm + per-token quantiser on host rows x [rows, cols] run on the device with the
 * model kernel (w NULL: quantise only). */
int llm_debug_norm_quant(int device, const float *x, const float *w, int rows, int cols, double eps,
                         int8_t *q, float *scales);
/* int8 GEMM C = A . B^T with the model's GEMM kernels.  splits >= 0: the warp-level kernel with
 * that split-K (0 = auto); -1: the tcgen05 kernel at the model's channel tile, -bn: tile width
 * bn; -(1000 + S): the tcgen05 kernel split over clusters of S = 2, 4 or 8 CTAs (the decode
 * projections' form).  The same for llm_debug_gemm_f16. */
int llm_debug_gemm_i8(int device, const int8_t *A, const int8_t *B, int M, int N, int K, int splits,
                      int32_t *C);
/* 16-bit GEMM (dtype LLM_DTYPE_F16 / BF16; inputs given as fp32 and rounded) -> fp32 C. */
int llm_debug_gemm_f16(int device, int dtype, const float *A, const float *B, int M, int N, int K,
                       int splits, float *C);
/* The device's exp2_det (the softmax and SwiGLU exponential: 2^x from round-to-nearest f32
 * steps, restated by the CPU oracle) on host values x[n]. */
int llm_debug_exp2(int device, const float *x, int n, float *out);
/* Read back cached K and V of (layer, seq, pos) as fp32 [kv_dim] each. */
int llm_debug_read_kv(llm_ctx *ctx, int layer, int seq, int pos, float *k, float *v);

#ifdef __cplusplus
}
#endif
#endif /* LLM_CUDA_H */
