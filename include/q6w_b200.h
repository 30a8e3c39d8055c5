/*
 * q6w_b200.h -- C ABI of the B200 (sm_100a) Q6W inference hot path.
 *
 * Q6W: signed int6 weights, one FP32 scale per output row, four values
 * packed low-bit-first into three bytes, rows stored row-major exactly as in
 * the reference file format (quantization/q6w_format.py:52-64, 101-227).
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer owned by the caller, unless
 *     the comment says "host".  Nothing here allocates device memory except
 *     the decode-graph cache kept inside a q6w_model (see q6w_generate_greedy).
 *   - Matrices are row-major; a Q6W matrix of [rows, cols] occupies
 *     rows*cols*3/4 bytes, cols % 4 == 0.
 *   - The last argument is the CUDA stream the work is enqueued on (pass
 *     0 for the legacy default stream).  Calls are asynchronous.
 *   - Every entry point returns Q6W_OK (0) or a negative status and never
 *     traps; q6w_last_error() gives a message for the calling host thread.
 *     This replaces the reference's silent early returns on bad arguments
 *     (scripts/neon_gqa_attention.c:15-19) and mirrors the status -1 of the
 *     HLS top (rtl/autonomous/tinyllm_autonomous.cpp:1093-1099).
 */
#ifndef Q6W_B200_H
#define Q6W_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define Q6W_API __attribute__((visibility("default")))
#else
#define Q6W_API
#endif

typedef struct CUstream_st* q6w_stream_t; /* == cudaStream_t */

enum {
  Q6W_OK = 0,
  Q6W_ERR_ARG = -1,      /* bad shape / null pointer / unsupported size   */
  Q6W_ERR_ALIGN = -2,    /* pointer not aligned as required               */
  Q6W_ERR_RANGE = -3,    /* token or position outside the model's range   */
  Q6W_ERR_CUDA = -4,     /* a CUDA runtime call failed                    */
  Q6W_ERR_DEVICE = -5    /* a kernel flagged bad device-side input        */
};

/* Message for the last failing call on this host thread ("" if none). */
Q6W_API const char* q6w_last_error(void);
/* ABI version, bumped on any incompatible change. */
Q6W_API int32_t q6w_abi_version(void);

/* ---- codec ------------------------------------------------------------- */

/* Decode packed Q6W rows to int8 codes in [-32, 31].
 * Replaces unpack_signed_int6 (quantization/q6w_format.py:67-81). */
Q6W_API int32_t q6w_unpack(const uint8_t* packed, int8_t* out, int64_t rows, int64_t cols,
                   q6w_stream_t stream);

/* out[r, c] = float(q[r, c]) * scales[r], one rounded FP32 product per
 * element -- bit-identical to the reference dequantization
 * (quantization/q6w_format.py:257-259). */
Q6W_API int32_t q6w_dequant(const uint8_t* packed, const float* scales, float* out, int64_t rows,
                    int64_t cols, q6w_stream_t stream);

/* The Q6W writer's row-wise quantization on the GPU: quantize_rows +
 * pack_signed_int6 (quantization/q6w_format.py:84-98, 52-64) with the same
 * FP32 operations, so codes and scales are bit-identical to the reference:
 * scales[r] = max|w[r,:]| / 31 (1.0 for an all-zero row), codes =
 * clamp(round-half-even(w / scale), -31, 31), packed into rows*cols*3/4
 * bytes.  weights [rows, cols] FP32 (finite; the caller checks), cols % 4 == 0.
 * row_err ([rows][3] FP64 scratch) and stats (3 FP64: max_abs_error,
 * mean_abs_error, rmse of q*scale - w) are optional (NULL); stats needs
 * row_err.  The statistics sum in FP64 in a fixed order, so they agree with
 * the reference's FP32 torch reductions to within their rounding. */
Q6W_API int32_t q6w_quantize_rows(const float* weights, int64_t rows, int64_t cols, uint8_t* packed,
                                  float* scales, double* row_err, double* stats, q6w_stream_t stream);

/* ---- linear ------------------------------------------------------------ */

/* y[n, rows] = x[n, cols] @ W^T with W = dequant(packed, scales): the
 * nn.Linear calls of the cached step (benchmarks/torch_benchmark.py:105-107,
 * 121, 123, 125) on Q6W weights, FP32 accumulation.  x and y are row-major
 * FP32, 4-byte aligned; n >= 0 (n == 0 is a no-op). */
Q6W_API int32_t q6w_linear(const uint8_t* packed, const float* scales, const float* x, float* y,
                   int64_t rows, int64_t cols, int64_t n, q6w_stream_t stream);

/* Workspace bytes q6w_linear_ex needs to run [rows, cols] x n on the tensor
 * cores, or 0 when that shape takes q6w_linear's FP32 kernels (n < 16, cols
 * not a multiple of 128 or above 8192, odd rows). */
Q6W_API size_t q6w_linear_workspace_bytes(int64_t rows, int64_t cols, int64_t n);

/* q6w_linear for batches -- the same nn.Linear calls (torch_benchmark.py:105-107,
 * 121, 123, 125) as a dense contraction on the tcgen05 tensor cores: x is
 * written once into the workspace as three bf16 parts (hi + mid + lo hold
 * every FP32 significand bit), the int6 codes are exact in bf16, products are
 * exact and accumulate in FP32 in tensor memory, and the row scale multiplies
 * each finished dot product.  The result agrees with the FP64 dequant-then-
 * matmul to within 1e-4 * sum_k |w_k x_k| per element (tensor-core
 * accumulation order; q6w_linear's FP32 kernels: 1e-5).  workspace: device,
 * 256-byte aligned, q6w_linear_workspace_bytes(rows, cols, n) bytes; its
 * first word is the error word q6w_workspace_status reads.  With a NULL
 * workspace, or a shape / alignment the tensor-core kernel does not take
 * (packed 16-byte aligned, x 16-byte, y 8-byte), this is q6w_linear. */
Q6W_API int32_t q6w_linear_ex(const uint8_t* packed, const float* scales, const float* x, float* y,
                              int64_t rows, int64_t cols, int64_t n, void* workspace,
                              size_t workspace_bytes, q6w_stream_t stream);

/* Vocab projection + greedy pick: logits = x @ W^T (optional, may be NULL)
 * and argmax[n] = first index of each row's maximum (torch.argmax), fused --
 * the tied-embedding classifier of torch_benchmark.py:125 with the greedy
 * sample_token of :148-150.  Replaces arm_neon_q6_vocab_sgemv_f32
 * (scripts/neon_q6_vocab.c:12-88) plus the host argmax.  `scratch` is
 * caller-owned device memory of >= 8*n bytes (8-byte aligned), overwritten.
 * Needs cols % 16 == 0, even rows, 16-byte aligned x. */
Q6W_API int32_t q6w_linear_argmax(const uint8_t* packed, const float* scales, const float* x,
                                  float* logits, int32_t* argmax, void* scratch,
                                  size_t scratch_bytes, int64_t rows, int64_t cols, int64_t n,
                                  q6w_stream_t stream);

/* q6w_linear_argmax without caller scratch: no counterpart in the reference.
 * For callers that cannot allocate device memory -- hosts binding this
 * library through a plain FFI (ctypes, JNI, cgo) that own no CUDA allocator,
 * and serving loops under a fixed device-memory budget where a per-call
 * cudaMalloc can fail and cudaFree synchronises the device.  The argmax keys
 * live in a library-owned device array of 32768 entries (256 KiB, held by
 * every GPU that loads the library until exit), so n <= 32768; larger n is
 * rejected with Q6W_ERR_ARG.  Allocates nothing.  The first call in each
 * CUDA context (each device's primary context, and again after a
 * cudaDeviceReset or when the caller makes another context current) looks
 * up the array's device address in that context (cudaGetSymbolAddress) and
 * caches it under the context's id; make that first call before any stream
 * capture.  All calls share the one array
 * (cleared at the start of each call): calls that overlap on the GPU, on
 * any streams, race and must be serialised by the caller. */
Q6W_API int32_t q6w_linear_argmax_noalloc(const uint8_t* packed, const float* scales,
                                          const float* x, float* logits, int32_t* argmax,
                                          int64_t rows, int64_t cols, int64_t n,
                                          q6w_stream_t stream);

/* out[s, :] = x[s, :] * (1 / sqrt(mean(x[s, :]^2) + eps)) * weight, for n
 * rows of `length` (torch_benchmark.py:22-24).  Replaces
 * arm_neon_rmsnorm_f32 (scripts/neon_rmsnorm.c:4-31). */
Q6W_API int32_t q6w_rmsnorm(const float* x, const float* weight, float* out, int32_t n,
                            int32_t length, float eps, q6w_stream_t stream);

/* Decode attention of n independent sequences over their FP32 caches
 * (torch_benchmark.py:113-119): for query head h (kv head h / groups_per_kv)
 *   out[s,h,:] = softmax_t(q[s,h,:] . K[s,t,kv,:] / sqrt(head_dim)) V[s,t,kv,:]
 * over t < lengths[s] (device int32, clamped to [0, max_len]; a length <= 0
 * gives zeros).  queries/output: [n, kv_heads*groups_per_kv, head_dim];
 * sequence s's keys/values start at keys/values + s*kv_seq_stride, laid out
 * [max_len, kv_heads, head_dim] (one layer of the cache).  Replaces
 * arm_neon_gqa_attention_f32 (scripts/neon_gqa_attention.c:11-95). */
Q6W_API int32_t q6w_gqa_attention(const float* queries, const float* keys, const float* values,
                                  float* output, const int32_t* lengths, int32_t n,
                                  int32_t kv_heads, int32_t groups_per_kv, int32_t head_dim,
                                  int32_t max_len, int64_t kv_seq_stride, q6w_stream_t stream);

/* ---- model ------------------------------------------------------------- */

typedef struct q6w_qmat {
  const uint8_t* packed; /* [rows, cols*3/4] bytes */
  const float* scales;   /* [rows] */
  int32_t rows, cols;
} q6w_qmat;

typedef struct q6w_layer_weights {
  q6w_qmat wq, wk, wv, wo, w1, w2, w3;
  const float* attention_norm; /* [dim] */
  const float* ffn_norm;       /* [dim] */
} q6w_layer_weights;

/* Model description: the manifest's model_args plus device pointers into the
 * uploaded Q6W image (the file's bytes, unchanged).  `layers` is a HOST array
 * of n_layers entries, copied by q6w_model_create. */
typedef struct q6w_model_desc {
  int32_t dim, n_layers, n_heads, n_kv_heads, vocab_size, hidden_dim, max_seq_len;
  float norm_eps;
  q6w_qmat tok_embeddings; /* [vocab, dim]; also the tied vocab head */
  const float* norm;       /* final RMSNorm weight [dim] */
  const float* rope_cos;   /* [max_seq_len, head_dim/2], host-built tables */
  const float* rope_sin;
  const q6w_layer_weights* layers; /* host */
} q6w_model_desc;

typedef struct q6w_model q6w_model;

/* Validate a description (shapes, alignment, supported head_dim) and create
 * a host-side handle.  Replaces CachedTransformer(args) +
 * load_state_dict (benchmarks/torch_benchmark.py:57-77). */
Q6W_API int32_t q6w_model_create(const q6w_model_desc* desc, q6w_model** out);
Q6W_API void q6w_model_destroy(q6w_model* model);

enum { Q6W_KV_F32 = 0, Q6W_KV_F16 = 1 };

/* Storage type of the KV cache for every later call on this model (default
 * Q6W_KV_F32).  With Q6W_KV_F16 the k_cache / v_cache arguments point at
 * IEEE half elements (same [.., max_seq_len, n_kv_heads, head_dim] layout
 * and element strides, half the bytes): the new K and V rows are rounded to
 * FP16 (nearest even) when written and widened exactly when read, and
 * attention computes in FP32 -- the reference's FP16-KV wrapper
 * (quantization/compare_kv_cache.py:15-72, FP16KVTransformer).  Available
 * for head dims 16 / 32 (up to 8 kv heads, groups of 1, 2 or 4) and 64 /
 * 128; the single-request cluster kernel is not used with it. */
Q6W_API int32_t q6w_model_set_kv_dtype(q6w_model* model, int32_t kv_dtype);

/* Workspace (device scratch, caller-allocated, 256-byte aligned) needed to
 * run up to max_seqs sequences per call. */
Q6W_API size_t q6w_workspace_bytes(const q6w_model* model, int32_t max_seqs);

/* KV cache: per sequence [n_layers, max_seq_len, n_kv_heads, head_dim] FP32,
 * the layout of CachedTransformer.new_cache (torch_benchmark.py:87-94).
 * Sequence s of a batch lives at k_cache + s * cache_seq_stride. */

/* One cached step of a single sequence: token id and position are host
 * values (validated here).  Writes the logits [vocab] row.
 * Replaces CachedTransformer.step (benchmarks/torch_benchmark.py:96-125). */
Q6W_API int32_t q6w_step(const q6w_model* model, int32_t token_id, int32_t position, float* k_cache,
                 float* v_cache, float* logits, void* workspace, size_t workspace_bytes,
                 q6w_stream_t stream);

/* One cached step of n_seqs independent sequences: tokens[s] at
 * positions[s] (device arrays).  logits is [n_seqs, vocab] or NULL; argmax
 * (first maximum, as torch.argmax) is [n_seqs] or NULL.  Out-of-range
 * tokens/positions are flagged on the device (see q6w_workspace_status) and
 * that sequence's writes are skipped. */
Q6W_API int32_t q6w_forward_batch(const q6w_model* model, int32_t n_seqs, const int32_t* tokens,
                          const int32_t* positions, float* k_cache, float* v_cache,
                          int64_t cache_seq_stride, float* logits, int32_t* argmax,
                          void* workspace, size_t workspace_bytes, q6w_stream_t stream);

/* Workspace bytes of q6w_prefill for n_prompts prompts of total_tokens tokens
 * together (0 if total_tokens is beyond the per-call limit of 2^22 rows). */
Q6W_API size_t q6w_prefill_workspace_bytes(const q6w_model* model, int32_t n_prompts, int64_t total_tokens);

/* Batched prefill of n_prompts independent prompts of ragged lengths:
 * prompts [n_prompts, prompt_stride] and prompt_lens [n_prompts] are device
 * arrays, 1 <= prompt_lens[i] <= max_prompt_len <= max_seq_len, and
 * total_tokens is the sum of the lengths.  Fills every prompt's K/V cache rows
 * 0..len-1 (prompt i at k_cache + i * cache_seq_stride) and writes the logits
 * of each prompt's last position, [n_prompts, vocab] (or NULL), and their
 * first-maximum argmax [n_prompts] (or NULL).  All prompt tokens run through
 * the layers at once (rows are tokens; each token attends over its prompt's
 * positions 0..j), so the result equals running CachedTransformer.step over
 * every prompt position in order, the prompt loop of
 * benchmarks/torch_benchmark.py:263-270.  Bad lengths, tokens or a total that
 * does not match the lengths are flagged on the device (q6w_workspace_status)
 * and the affected rows write nothing. */
Q6W_API int32_t q6w_prefill(const q6w_model* model, int32_t n_prompts, const int32_t* prompts,
                    const int32_t* prompt_lens, int32_t prompt_stride, int32_t max_prompt_len,
                    int64_t total_tokens, float* k_cache, float* v_cache, int64_t cache_seq_stride,
                    float* last_logits, int32_t* last_argmax, void* workspace, size_t workspace_bytes,
                    q6w_stream_t stream);

/* The non-cached forward with targets -- Transformer.forward(tokens, targets)
 * of training/model.py:249-269 -- on ragged prompts (arguments and KV-cache
 * filling as q6w_prefill, same workspace): logits [total_tokens, vocab] of
 * every position (row off_i + j for position j of prompt i, off_i the sum of
 * the earlier prompts' lengths; 16-byte aligned), and when targets
 * [n_prompts, prompt_stride] (device int32) is given, *loss (device, one
 * float) = the mean cross entropy over the positions whose target is not -1
 * (F.cross_entropy(..., ignore_index=-1); NaN if every target is -1).  A
 * target outside [0, vocab) other than -1 is flagged on the device
 * (q6w_workspace_status) and that position is not counted.  targets and loss
 * are both NULL or both set. */
Q6W_API int32_t q6w_forward_all(const q6w_model* model, int32_t n_prompts, const int32_t* prompts,
                                const int32_t* prompt_lens, int32_t prompt_stride, int32_t max_prompt_len,
                                int64_t total_tokens, float* k_cache, float* v_cache, int64_t cache_seq_stride,
                                float* logits, const int32_t* targets, float* loss, void* workspace,
                                size_t workspace_bytes, q6w_stream_t stream);

/* Greedy generation of n_seqs independent requests, entirely on the device:
 * token-by-token prefill of each (ragged) prompt, then greedy decode with
 * the reference's stop contract -- stop ids masked to -inf while fewer than
 * min_new_tokens tokens exist, first-maximum argmax, and a stop id picked
 * afterwards ends the request without being appended
 * (benchmarks/torch_benchmark.py:233-296 at temperature 0;
 *  scripts/prepare_e2e.py:121-143;
 *  rtl/autonomous/tinyllm_autonomous.cpp:1114-1150).
 * One CUDA graph per step is replayed max_prompt_len + new_tokens - 1 times
 * with no host synchronisation; the graph is cached in the model handle. */
typedef struct q6w_greedy_args {
  int32_t n_seqs;
  const int32_t* prompts;     /* [n_seqs, prompt_stride] */
  const int32_t* prompt_lens; /* [n_seqs], each in [1, max_prompt_len] */
  int32_t prompt_stride;
  int32_t max_prompt_len;     /* host value: max of prompt_lens */
  int32_t new_tokens;         /* >= 1; max_prompt_len + new_tokens - 1 <= max_seq_len */
  const int32_t* stop_ids;    /* host array of n_stop ids (copied), may be NULL */
  int32_t n_stop;             /* 0..8 */
  int32_t min_new_tokens;     /* 0..new_tokens */
  int32_t* sampled;           /* [n_seqs, new_tokens]: every argmax pick, incl. a final stop id */
  int32_t* n_sampled;         /* [n_seqs] */
  int32_t* stop_reason;       /* [n_seqs]: the stop id that ended the request, or -1 */
  float* k_cache;
  float* v_cache;
  int64_t cache_seq_stride;
  float* step_logits;         /* [n_seqs, new_tokens, vocab] raw logits of each pick, or NULL */
  void* prefill_event;        /* cudaEvent_t recorded after the first max_prompt_len steps, or NULL */
} q6w_greedy_args;

Q6W_API int32_t q6w_generate_greedy(q6w_model* model, const q6w_greedy_args* args, void* workspace,
                            size_t workspace_bytes, q6w_stream_t stream);

/* Sampling and logit shaping of torch_benchmark.generate
 * (benchmarks/torch_benchmark.py:133-230, applied as in :272-286).  Values
 * the reference applies to FP32 logits (temperature, repetition_penalty,
 * stop_token_bias) act as their FP32 roundings, as torch applies a Python
 * float to a float32 tensor; top_p is compared in FP64 as in the reference. */
typedef struct q6w_sample_args {
  float temperature;             /* 0: the first maximum of the shaped logits (greedy) */
  double top_p;                  /* nucleus mass; <= 0 or >= 1: scan over every token */
  float repetition_penalty;      /* 1: off; else logits of generated tokens: l < 0 ? l * p : l / p */
  int32_t no_repeat_ngram_size;  /* 0: off */
  float stop_token_bias;         /* added to the stop ids' logits from decode index stop_token_bias_after on */
  int32_t stop_token_bias_after; /* the reference's default is min_new_tokens */
  const uint64_t* seeds;         /* [n_seqs] device array: XorShift64 seed of each request (temperature > 0) */
} q6w_sample_args;

/* q6w_generate_greedy with the reference's sampler: with `sampling` NULL (or
 * temperature 0 and no shaping) this is the greedy loop; otherwise every
 * step's logits row goes through the repetition penalty, n-gram blocking,
 * stop-id masking (before min_new_tokens) or bias (from
 * stop_token_bias_after on), and temperature / top-p sampling with one
 * XorShift64 generator per request seeded from `seeds`, all on the device
 * in the same CUDA graph step.  The workspace is q6w_workspace_bytes (it
 * includes the sampler's [n, vocab] logits and generator states).  A picked
 * stop id ends the request (not appended), as in generate. */
Q6W_API int32_t q6w_generate(q6w_model* model, const q6w_greedy_args* args, const q6w_sample_args* sampling,
                             void* workspace, size_t workspace_bytes, q6w_stream_t stream);

/* The sampler alone, on n rows of logits (row i at logits + i * ld, vocab
 * columns; not modified): replaces the reference's per-step host code of
 * generate (:272-285) for callers that compute logits themselves.
 * history [n, history_ld] holds each row's generated tokens (history_len[i]
 * of them, which is also the decode index for stop masking and bias);
 * rng_state [n] holds each row's XorShift64 state (a new generator's state
 * is its seed) and is advanced when a coin is drawn; stop_ids is a host
 * array of n_stop (<= 8) ids.  tokens [n] receives the picks.  Device
 * arrays unless marked host; vocab <= 32768. */
Q6W_API int32_t q6w_sample(const float* logits, int64_t ld, int32_t n, int32_t vocab, const int32_t* history,
                           int64_t history_ld, const int32_t* history_len, uint64_t* rng_state,
                           const q6w_sample_args* sampling, const int32_t* stop_ids, int32_t n_stop,
                           int32_t min_new_tokens, int32_t* tokens, q6w_stream_t stream);

/* Synchronise `stream` and report device-side errors recorded in the
 * workspace since the last call (then clear them): Q6W_OK, or Q6W_ERR_DEVICE
 * for rejected input (bit 0) or a device wait that ran out of time (bit 2). */
Q6W_API int32_t q6w_workspace_status(void* workspace, q6w_stream_t stream);

/* Diagnostic with no counterpart in the reference: one CTA waits on an
 * mbarrier that no thread arrives at, through the bounded-wait routine every
 * pipeline wait of this library uses, limited to wait_cycles SM clock cycles
 * (1 .. 2^31; the pipelines use about 4e9).  When the wait runs out the CTA
 * sets the timeout bit in the workspace's error word and returns, so the
 * context stays usable; q6w_workspace_status then reports Q6W_ERR_DEVICE.
 * Lets a deployment check on its own GPU that a stalled pipeline ends with a
 * status instead of a hang. */
Q6W_API int32_t q6w_selftest_wait_timeout(void* workspace, int64_t wait_cycles, q6w_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* Q6W_B200_H */
