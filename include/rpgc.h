/* rpgc.h -- the thin C-ABI CUDA layer under the RPGBarEngine host (B200, sm_100a).
 *
 * This is the drop-in boundary for the token loop: plain C types, handles and
 * pointers, no C++ or torch types, no exceptions.  Every call returns a status
 * (RPGC_OK = 0, negative = error) or a handle (< 0 = error); the message of
 * the last failure on the calling thread is rpgc_last_error(), the same
 * convention as the reference ABI (include/rpg_engine.h:48-52,
 * src/engine.cc:175-191).
 *
 * The layer replaces the reference's internal C++ seam between the host and
 * the token loop (src/qwen3.h:83-142, src/kv_cache.h:35-82,
 * src/model.h:62-92, src/matmul.h:35-64, src/quant.h:65).  The host keeps the
 * text side (tokenizer, chat template, tool parsing) and calls this layer with
 * token ids.
 *
 * Ownership: the caller owns host buffers; the layer owns device memory.  A
 * session owns one CUDA stream; calls on different sessions may run from
 * different host threads, one call at a time per session
 * (include/rpg_engine.h:13-14).  Kernel-level entry points take device
 * pointers and a cudaStream_t passed as void* (NULL = the legacy default
 * stream).
 */
#ifndef RPGC_H
#define RPGC_H

#include <stdint.h>

#if defined(__GNUC__)
#define RPGC_API __attribute__((visibility("default")))
#else
#define RPGC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------- status codes */
#define RPGC_OK 0
#define RPGC_E_ARG (-1)          /* bad argument / unsupported type or shape */
#define RPGC_E_CUDA (-2)         /* CUDA runtime error */
#define RPGC_E_OOM (-3)          /* device allocation failed */
#define RPGC_E_STATE (-4)        /* invalid handle or call order */
#define RPGC_E_CONTEXT_FULL (-5) /* KV cache would overflow (src/qwen3.cc:341-344) */
#define RPGC_E_TIMEOUT (-6)      /* a bounded device wait gave up */
#define RPGC_E_IO (-7)           /* GGUF file could not be read */

/* ggml type ids (src/quant.h:22-38); the kernels take F32, Q8_0, Q4_K, Q6_K. */
#define RPGC_F32 0u
#define RPGC_F16 1u
#define RPGC_Q8_0 8u
#define RPGC_Q4_K 12u
#define RPGC_Q6_K 14u

/* One GGUF tensor: raw block bytes, dims[0] fastest (src/gguf.h:30-42). */
typedef struct rpgc_tensor {
  const char* name;
  uint32_t type;
  int32_t n_dims;
  int64_t dims[4];
  const void* data; /* host pointer to the raw bytes */
  int64_t n_bytes;
} rpgc_tensor;

/* Model hyper-parameters (src/model.h:30-58).  max_pos caps the RoPE table
 * at min(max_pos, context_length) positions (src/model.cc:122-145). */
typedef struct rpgc_model_config {
  int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
  int32_t context_length, max_pos;
  float rope_theta, rms_eps;
} rpgc_model_config;

/* Decode-loop options (src/qwen3.h:113-126, src/sampler.h:35-44).
 * temperature <= 0 is greedy; top_k only applies when 1 < top_k < vocab;
 * top_p only when 0 < top_p < 1; at most RPGC_MAX_STOP stop ids. */
#define RPGC_MAX_STOP 16
typedef struct rpgc_gen_opts {
  int32_t max_tokens;
  const int32_t* stop_ids;
  int32_t n_stop;
  float temperature;
  int32_t top_k;
  float top_p;
  uint64_t seed;
} rpgc_gen_opts;

/* ------------------------------------------------------------- library */
RPGC_API const char* rpgc_version(void);
/* Kernels the library has enqueued on any device since it was loaded (a
 * decode-step graph replay counts each kernel in it).  Instrumentation for
 * benchmarks; no counterpart in the reference. */
RPGC_API int64_t rpgc_kernel_launches(void);
/* Thread-local; valid until the next call on this thread; do not free
 * (src/common.cc:11, 54-56). */
RPGC_API const char* rpgc_last_error(void);
RPGC_API int rpgc_device_count(void);

/* --------------------------------------------------------------- model */
/* Replaces Model::Load (src/model.cc:147-281): shape-checked Qwen3 tensor
 * table, raw blocks copied to HBM unchanged, F32 norms, RoPE table built on
 * the host in double and rounded to float.  Returns a model handle (>= 1). */
RPGC_API int32_t rpgc_model_upload(int device, const rpgc_model_config* cfg,
                                   const rpgc_tensor* tensors, int32_t n_tensors);
/* Parses a GGUF v1-v3 file (src/gguf.cc:69-160), reads the qwen3.*
 * hyper-parameters (src/model.cc:159-211) and uploads it. */
RPGC_API int32_t rpgc_model_load_gguf(int device, const char* path, int32_t max_pos);
/* Tensor parallelism (the 8B shape: row-split q/k/v/gate/up and untied
 * output, column-split o and down).  Prefill: one NCCL all-reduce after each
 * column-split matmul, the logits' vocabulary slices all-gathered.  Decode:
 * the persistent step kernel of every rank stores its partial rows into every
 * rank's inbox over peer memory (no collective call per token).  One process
 * per GPU: one rank calls rpgc_tp_id (a 128-byte NCCL unique id), every rank
 * passes the same bytes with its rank to rpgc_model_upload_tp and then makes
 * the same session calls in the same order (each holds collectives or
 * cross-rank waits).  The tensor table is the whole model's; each rank
 * uploads its shard.  Needs libnccl.so.2 at run time. */
RPGC_API int rpgc_tp_id(void* id, int64_t bytes);
/* One rank's shard of a tensor-parallel model: its head, kv-head and
 * intermediate counts, the row ranges [begin, end) it holds of attn_q,
 * attn_k / attn_v, ffn_gate / ffn_up and the untied output (vocabulary), and
 * the column ranges of attn_output and ffn_down.  Checks what
 * rpgc_model_upload_tp checks of the shapes (every count divides by world);
 * needs no device.  rpgc_model_upload_tp takes its ranges from here. */
typedef struct rpgc_tp_shard {
  int32_t n_heads, n_kv_heads, intermediate;
  int64_t q_rows[2], kv_rows[2], ffn_rows[2], vocab_rows[2];
  int64_t o_cols[2], down_cols[2];
} rpgc_tp_shard;
RPGC_API int rpgc_tp_shard_of(const rpgc_model_config* cfg, int32_t rank, int32_t world, rpgc_tp_shard* out);
RPGC_API int32_t rpgc_model_upload_tp(int device, const rpgc_model_config* cfg,
                                      const rpgc_tensor* tensors, int32_t n_tensors, int32_t rank,
                                      int32_t world, const void* id);
/* The whole model's configuration (also for a tensor-parallel shard). */
RPGC_API int rpgc_model_get_config(int32_t model, rpgc_model_config* out);
/* Raw weight bytes resident in HBM (src/model.h:139-143). */
RPGC_API int64_t rpgc_model_weight_bytes(int32_t model);
/* Frees the model and every session on it (src/engine.cc:246-257). */
RPGC_API int rpgc_model_free(int32_t model);

/* ------------------------------------------------------------- session */
/* Device KV cache [n_layers][n_kv_heads][max_seq][head_dim] fp32 for K and
 * V, zero-initialised (src/kv_cache.h:35-82, src/kv_cache.cc:5-33). */
RPGC_API int32_t rpgc_session_create(int32_t model, int32_t max_seq);
RPGC_API int rpgc_session_destroy(int32_t session);
RPGC_API int64_t rpgc_session_len(int32_t session);
/* Prefix reuse: positions [0, len) stay valid (src/engine.cc:425-431,
 * src/kv_cache.h:63-69).  Invalidates the pending logits. */
RPGC_API int rpgc_session_set_len(int32_t session, int64_t len);
/* Shared-prefix reuse across sessions of one model: copies KV positions
 * [0, n) of every layer and kv head from session src into session dst on the
 * device and sets dst's length to n (pending logits invalidated, so a
 * rpgc_forward of the rest follows).  The reference reuses a prefix only
 * within one session (LCP, src/engine.cc:383-448); this lets many sessions
 * that open with the same tokens (a shared system prompt) compute them once.
 * n <= rpgc_session_len(src); n > dst's capacity is RPGC_E_CONTEXT_FULL. */
RPGC_API int rpgc_session_copy_prefix(int32_t dst, int32_t src, int64_t n);
/* cudaStream_t of the session, as void* (for event timing). */
RPGC_API void* rpgc_session_stream(int32_t session);
/* Copies the cache to host arrays of n_layers*n_kv_heads*max_seq*head_dim
 * floats each (either may be NULL). */
RPGC_API int rpgc_session_read_kv(int32_t session, float* k, float* v);

/* ForwardFull / ForwardStep (src/qwen3.cc:208-300): appends n tokens at
 * pos0 = len, writes K/V, len += n.  last_logits (vocab floats) receives the
 * last row; all_logits (n*vocab floats) every row; either may be NULL.  The
 * last row also stays on the device as the next rpgc_generate's input. */
RPGC_API int rpgc_forward(int32_t session, const int32_t* ids, int64_t n, float* last_logits,
                          float* all_logits);
/* Generate (src/qwen3.cc:302-355): device-resident decode loop starting from
 * the pending last-row logits; each picked token (the stop token included) is
 * forwarded, so len grows by *n_out.  u = CounterUniform(seed, len) per step
 * (src/sampler.cc:24-34).  out_ids needs max_tokens slots.  With batching on
 * for the session's model (rpgc_model_set_batching), concurrent calls from
 * other threads may decode together with this one; the call still returns
 * only its own session's ids and status. */
RPGC_API int rpgc_generate(int32_t session, const rpgc_gen_opts* opts, int32_t* out_ids,
                           int32_t* n_out);
/* Same two calls with device-resident ids / results and no host transfer of
 * logits (the benchmark's kernel-only leg).  ids_dev: n int32 on the device;
 * out_ids_dev: max_tokens int32 on the device; n_out stays on the device too
 * (n_out_dev, one int32).  Asynchronous on the session stream. */
/* The ids must be on the device before the session's stream reads them (the
 * caller orders its own copy, e.g. by synchronising).  They are not checked on
 * the host: an id outside the vocabulary embeds as zeros and the next
 * rpgc_session_sync returns RPGC_E_ARG. */
RPGC_API int rpgc_forward_device(int32_t session, const int32_t* ids_dev, int64_t n);
RPGC_API int rpgc_generate_device(int32_t session, const rpgc_gen_opts* opts,
                                  int32_t* out_ids_dev, int32_t* n_out_dev);
/* Batched multi-session decode: max_tokens steps that each decode one token
 * for every one of the n sessions (1 .. 256, one model, each with pending
 * logits and room for max_tokens more positions) at once, with the same
 * options for all (each session keeps its own position, stop state and
 * seeded draws, as rpgc_generate would give it).  The reference decodes one
 * session at a time (Generate, src/qwen3.cc:302-355, per session); here the
 * weight stream is shared: the matmuls run on the tensor cores over the n
 * session rows, the attention reads each session's own cache.  out_ids holds
 * n x max_tokens ids (row i = session i, n_out[i] valid); afterwards each
 * session is as after rpgc_generate.  Each session is finished with its own
 * outcome; the call returns the first failure (a failed session's n_out is
 * 0 and its length unchanged).  Not for tensor-parallel models.  Steps replay
 * a CUDA graph of one step, captured on the first session's stream by the
 * first batch of each size (the model keeps the graphs and the batch buffers
 * between batches), so that stream must not be under stream capture. */
RPGC_API int rpgc_generate_batch(const int32_t* sessions, int32_t n, const rpgc_gen_opts* opts,
                                 int32_t* out_ids, int32_t* n_out);
/* Batching behind rpgc_generate (no counterpart in the reference, whose
 * engine generates for one session per call, src/engine.cc:349-515): with
 * max_batch >= 2, rpgc_generate calls on sessions of this model made
 * concurrently from different host threads are gathered, up to max_batch
 * sessions, waiting at most window_us microseconds for more once the first
 * arrives, and decoded as one batch (as rpgc_generate_batch, each call with
 * its own options, stop ids and max_tokens).  Each call returns when its
 * batch ends, with its own ids and status; a call that arrives while a
 * batch runs joins the next one.  A call alone after the window decodes
 * unbatched: with batching on, a call that no other caller joins waits up to
 * window_us before it starts (the price of the gathering; keep window_us
 * small, or leave batching off for a single caller).  Calls that are not eligible (no pending logits, less room
 * than max_tokens, invalid options) run unbatched and report their errors
 * as before.  Batched tokens match an unbatched call's within the parity
 * tolerance (the matmuls run on the tensor cores).  max_batch 0 or 1 turns
 * batching off (the default); max_batch 2 .. 256, window_us 0 .. 1000000.
 * Not for tensor-parallel models. */
RPGC_API int rpgc_model_set_batching(int32_t model, int32_t max_batch, int32_t window_us);
/* Batches of two or more sessions run so far for this model, and the
 * rpgc_generate calls they served. */
RPGC_API int rpgc_model_batching_stats(int32_t model, int64_t* batches, int64_t* requests);
/* Test hook, no counterpart in the reference: in the next batched decode (on
 * any model), the session at position `index` of the batch has its
 * attention thread blocks of layer 0 wait, at every step, on a barrier that
 * nothing completes.  The bounded wait gives up and flags that session only:
 * its call (or its entry of rpgc_generate_batch) fails with RPGC_E_TIMEOUT
 * while the other sessions complete.  -1 clears a pending stall.  For tests of
 * the failure path; nothing else sets it. */
RPGC_API int rpgc_test_stall_next_batch(int32_t index);
RPGC_API int rpgc_session_sync(int32_t session);

/* ------------------------------------------- token-level engine sessions */
/* The reference's public session calls (rpg_engine_session_create / _reset /
 * _destroy / _generate, include/rpg_engine.h:52-117, src/engine.cc:259-515)
 * with the text side left to the host: the host renders the chat template,
 * tokenises, and passes each turn's whole prompt as token ids (with the BOS
 * id when the model adds one); it receives the completion as token ids and
 * decodes and parses it.  Between the two, the engine does what the
 * reference does: longest-common-prefix reuse of the session's cache, the
 * capacity check before the cache is touched, reset on a failed forward,
 * the model's and the caller's stop ids, sampling with top_k 0 and top_p
 * 0.95, and the finish reason by tokens.  Handles start at 1 and are never
 * reused; destroying an unknown handle is a no-op; one generate at a time
 * per session (the host serialises, include/rpg_engine.h:13-14). */
typedef struct rpgc_engine_session_opts {
  int32_t max_seq;        /* cache positions; 0: the model's RoPE positions (src/engine.cc:264-268) */
  int32_t max_tokens;     /* default per request; 0: 256; narrowed to max_seq - 1 (:272-286) */
  float temperature;      /* default; clamped to [0, 2], 0 = greedy (:295-303) */
  uint64_t seed;          /* default seed (:304-305) */
  const int32_t* stop_ids; /* the session's single-token stop strings, as ids (:288-293, 456) */
  int32_t n_stop;
} rpgc_engine_session_opts;

typedef struct rpgc_engine_request {
  int32_t max_tokens;      /* <= 0: the session's (src/engine.cc:399-400) */
  int32_t set_temperature; /* nonzero: temperature below, else the session's (:404-410) */
  float temperature;       /* clamped to [0, 2] */
  int32_t set_seed;        /* nonzero: seed below, else the session's (:411) */
  uint64_t seed;
  const int32_t* stop_ids; /* the request's single-token stop strings, as ids (:455) */
  int32_t n_stop;
} rpgc_engine_request;

#define RPGC_FINISH_STOP 0   /* a stop id ended it, or it ended short of max_tokens */
#define RPGC_FINISH_LENGTH 1 /* max_tokens ids and the last is not a stop id */
typedef struct rpgc_engine_result {
  int32_t n_out;         /* generated ids (usage.completion_tokens) */
  int32_t finish;        /* RPGC_FINISH_*, by tokens (src/engine.cc:477-487); "tool_calls" and a
                            completion cut inside a tool call or think block are the host
                            parser's call */
  int64_t prompt_tokens; /* usage.prompt_tokens */
  int64_t reused;        /* prompt positions served from the cache (the common prefix) */
} rpgc_engine_result;

/* rpg_engine_session_create (src/engine.cc:259-308) on a model of this
 * library; opts NULL = every default.  Returns a handle >= 1. */
RPGC_API int32_t rpgc_engine_session_create(int32_t model, const rpgc_engine_session_opts* opts);
/* rpg_engine_session_destroy (src/engine.cc:310-323). */
RPGC_API int rpgc_engine_session_destroy(int32_t session);
/* rpg_engine_session_reset (src/engine.cc:336-346): length 0, memory kept. */
RPGC_API int rpgc_engine_session_reset(int32_t session);
/* The ids the session's cache holds (prompt and generated ids of its turns
 * so far): copies up to cap of them into ids (may be NULL), returns how many
 * there are (< 0: error). */
RPGC_API int64_t rpgc_engine_session_cached(int32_t session, int32_t* ids, int64_t cap);
/* rpg_engine_generate (src/engine.cc:349-515) on token ids: prompt ids[0, n)
 * is the whole conversation so far, rendered and tokenised by the host; req
 * NULL = the session's defaults.  out_ids needs room for max_tokens ids.  A
 * prompt + max_tokens + 4 beyond the session's positions is
 * RPGC_E_CONTEXT_FULL with the cache untouched; a forward that fails resets
 * the session's cache. */
RPGC_API int rpgc_engine_generate(int32_t session, const int32_t* ids, int64_t n,
                                  const rpgc_engine_request* req, int32_t* out_ids, int32_t out_cap,
                                  rpgc_engine_result* res);
/* The model's end-of-sequence and <|im_end|> ids, the engine's model-level
 * stop ids (src/model.cc:187, src/engine.cc:451-454): read from a GGUF's
 * tokenizer.ggml.eos_token_id and vocabulary by rpgc_model_load_gguf, -1
 * (none) for a model uploaded from a tensor table until set here. */
RPGC_API int rpgc_model_set_special_ids(int32_t model, int32_t eos_id, int32_t im_end_id);
RPGC_API int rpgc_model_special_ids(int32_t model, int32_t* eos_id, int32_t* im_end_id);

/* ------------------------------------------------ kernel entry points */
/* DequantizeRow (src/quant.h:65) over rows*cols elements, bit-exact. */
RPGC_API int rpgc_dequantize_rows(uint32_t type, const void* w, int64_t rows, int64_t cols,
                                  float* out, void* stream);
/* One fused-dequant matrix-vector product: y[r] = dot(x, W[r])
 * (QuantMatrix::MatVec, src/model.cc:23-30; DotRowQuant, src/matmul.h:35).
 * w must be 16-byte aligned and readable up to the next 16-byte boundary
 * past its last byte; cols must be a multiple of 64. */
RPGC_API int rpgc_matvec(uint32_t type, const void* w, int64_t rows, int64_t cols,
                         const float* x, float* y, void* stream);
/* OUT[t*rows + r] = dot(X[t], W[r]) (QuantMatrix::MatMulBatch,
 * src/model.cc:39-69; MatMulBlocked, src/matmul.h:55).  n == 1 takes the
 * decode kernel, n > 1 the prefill kernel.  X must be 16-byte aligned. */
RPGC_API int rpgc_matmul(uint32_t type, const void* w, int64_t rows, int64_t cols,
                         const float* X, int64_t n, float* OUT, void* stream);
/* AttentionFromCache for one query token (src/qwen3.cc:79-117, seq = 1):
 * q holds n_heads*head_dim floats (already QK-normed and rotated), the caches
 * are one layer in the KvCache layout [n_kv_heads][max_seq][head_dim]
 * (src/kv_cache.cc:29-33), 16-byte aligned; keys [0, pos] are read; out
 * receives n_heads*head_dim floats.  The positions are split over one
 * thread-block cluster per kv head that merges its splits on chip: no scratch
 * memory.  head_dim must be 128 and n_heads/n_kv_heads 1, 2, 4 or 8. */
RPGC_API int rpgc_attention_decode(const float* q, const float* k_cache, const float* v_cache,
                                   int64_t max_seq, int32_t n_heads, int32_t n_kv_heads,
                                   int32_t head_dim, int64_t pos, float* out, void* stream);
/* rpgc_matmul that allocates nothing.  No counterpart in the reference.
 * For callers that cannot let this library allocate device memory: a host
 * whose GPU heap belongs to another runtime (a game engine that forbids
 * foreign cudaMalloc/cudaFree), or a path where an allocation may block or
 * fail.  Same arguments and results as rpgc_matmul; the tensor-core kernels'
 * scratch (fp16 split of X, row scales, split-K partial sums) is a fixed
 * 32 MiB device array of the library on every GPU that loads it (held until
 * exit) instead of memory allocated per call.  n x cols beyond what fits
 * (about 4*n*cols + 36864*n bytes) is rejected with RPGC_E_ARG and a message.
 * Every call looks the array's address up on the current device (an address
 * kept from an earlier call could be stale after a device reset); the first
 * call on a device may load the library's device code there, so it should
 * come before any stream capture on that device.  All
 * calls on a device share the array: calls that overlap on the GPU race, so
 * order them on one stream or synchronise between them. */
RPGC_API int rpgc_matmul_noalloc(uint32_t type, const void* w, int64_t rows, int64_t cols,
                                 const float* X, int64_t n, float* OUT, void* stream);
/* SampleToken / ArgMax on device logits (src/sampler.cc:96-112,
 * src/kernels.h:42-52); *token_dev receives the id. */
RPGC_API int rpgc_sample(const float* logits, int64_t n, float temperature, int32_t top_k,
                         float top_p, float u, int32_t* token_dev, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* RPGC_H */
