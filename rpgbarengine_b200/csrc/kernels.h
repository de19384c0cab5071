// kernels.h -- host-side launch interface of the sm_100a kernels (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rpgc {

// Decode-loop state living in device memory, so that one captured CUDA graph
// serves every step (the position and the stop status are read in-kernel).
// DecodeState::error flags besides the bounded-wait timeout (common.cuh)
constexpr int32_t kErrBadToken = 2;  // a device-resident token id outside the embedding table

struct DecodeState {
  int32_t pos;        // KV length = position of the token being forwarded
  int32_t start_pos;  // KV length when generation started
  int32_t active;     // 0: this step does nothing (generation finished)
  int32_t done;       // set once a stop id / max_tokens was reached
  int32_t n_gen;      // tokens produced so far
  int32_t max_tokens;
  int32_t n_stop;
  int32_t top_k;
  int32_t token;      // token being forwarded this step
  float temperature;
  float top_p;
  uint64_t seed;
  int32_t stop_ids[16];
  int32_t error;      // kernel error flags (bounded waits)
  int32_t cand_ok;    // the pending logits' candidates (LogitCands): 0 none, 1 argmax, 2 argmax + top list
};

// Candidates the decode step's lm_head phase leaves beside the logits, per
// CTA of the step kernel (its contiguous vocabulary rows): the first index of
// its maximum, and (when sampling with 1 < top_k <= kCandK) its kCandK largest
// logits, ties to the lower index, listed in index order (index -1: padding
// for a CTA with fewer rows).  The sampler takes the argmax or the top-k
// survivors from them instead of sweeping the whole vocabulary.
constexpr int32_t kCandK = 32;
struct LogitCands {
  float* val;      // [ctas][kCandK] raw logits
  int32_t* idx;    // [ctas][kCandK]
  float* max_val;  // [ctas]
  int32_t* max_idx;
  int32_t ctas;
};

// ------------------------------------------------------------------ GEMV
enum GemvMode : int32_t { kStore = 0, kAdd = 1, kSwiGLU = 2 };

struct GemvSeg {
  const uint8_t* w;  // raw row-major blocks
  float* out;        // rows outputs
  int64_t rows;
  int64_t row_bytes;
  uint32_t type;
  int32_t mode;      // kSwiGLU: this seg is the gate, seg+1 the up projection
};

// Rows of the next matrix-vector launch to prefetch into L2: CTA b of this
// launch prefetches the first pf_bytes of the rows CTA b of the next launch
// owns (the same balanced split over the grid).
struct GemvPrefetch {
  const uint8_t* w;
  int64_t rows;
  int64_t row_bytes;
};

struct GemvArgs {
  GemvSeg seg[4];
  int32_t nseg;
  GemvPrefetch pf[4];
  int32_t npf;
  int32_t pf_bytes;
  int32_t K;              // shared input length (multiple of 64)
  const float* x;         // input [K]
  const float* norm_w;    // optional RMSNorm gain applied to x first
  float eps;
  const int32_t* active;  // optional: skip when *active == 0
  int32_t* err;           // optional error flags
};

// Library-wide count of kernels enqueued (instrumentation for benchmarks):
// every launch function adds the kernels it enqueued.
void count_launches(int64_t k);
int64_t launches_enqueued();

// Launch y = W x over up to 4 segments sharing x (decode, batch 1).  Weight
// bytes up to the next 16-byte boundary past each segment's last row are
// read (and ignored).
cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t s, bool pdl);
// Whether gemv_launch takes input length K (a multiple of 128; with an
// RMSNorm gain when norm is set).
bool gemv_supported(int64_t K, bool norm);

// Tensor parallelism: rows of logits gathered rank-major ([world][nc][vl])
// interleaved into [nc][world * vl].
cudaError_t gather_vocab_launch(const float* src, int world, int64_t nc, int64_t vl, float* dst,
                                cudaStream_t s);

// ------------------------------------------------- persistent decode step
// One matrix-vector phase of the step (up to three segments sharing x).
struct StepGemv {
  GemvSeg seg[3];
  int32_t nseg;
  int32_t K;
  const float* x;
  const float* norm_w;  // optional RMSNorm gain
};
// One decode-attention phase (one layer, the token at state->pos).
struct StepAttn {
  const float* q;       // [n_heads][128] raw projections
  const float* k_new;   // [n_kv][128]
  const float* v_new;
  const float* q_norm;  // [128]
  const float* k_norm;
  float* kc;            // this layer's caches [n_kv][max_seq][128]
  float* vc;
  float* out;           // [n_heads][128]
};
struct StepPhaseIn {
  int32_t kind;  // 0 matrix-vector, 1 attention
  StepGemv g;
  StepAttn a;
  int32_t cand;  // the lm_head phase: leave LogitCands of its output rows
  // Tensor parallelism (a plan created with a StepTp): the input is the
  // residual plus the sum of every rank's partial rows of the last exchange
  // (x_sum), and / or the outputs go to every rank (xchg 1: partial rows into
  // each rank's inbox, summed by the next phase; 2: rows into each rank's
  // copy of the whole output at this rank's row offset).
  int32_t x_sum;
  int32_t xchg;
};
// Tensor-parallel shape of a step plan: this rank, the rank count, the
// residual width (the rows every exchange carries) and, for the gathered
// last phase, this rank's row offset in the whole output.
struct StepTp {
  int32_t rank, world;
  int32_t hidden;
  int64_t gather_offset;
};
constexpr int kMaxTp = 8;
struct StepPlan;
// Plans the step's phases for `device` (shapes, ring, shared memory) and
// uploads the phase table; fails (cudaErrorInvalidValue) for block types or
// shapes the step kernel does not take, so the caller keeps per-launch kernels.
cudaError_t step_plan_create(const StepPhaseIn* in, int n, int n_heads, int n_kv, int64_t max_seq,
                             int device, StepPlan** out, const StepTp* tp = nullptr);
// Tensor-parallel plans: the device allocation every rank must map (the
// exchange inboxes and counters), and the binding of every rank's mapping of
// it and of its whole-output buffer (indexed by rank, this rank's own
// included); the plan launches only after the binding.
void* step_plan_tp_arena(const StepPlan* p);
cudaError_t step_plan_tp_bind(StepPlan* p, void* const* arenas, float* const* outputs);
void step_plan_free(StepPlan* p);
int step_plan_splits(const StepPlan* p);
int step_plan_grid(const StepPlan* p);
// Attention partial scratch (floats) of a plan.
size_t step_part_floats(const StepPlan* p);
// One decode step: every phase of the plan in one cooperative launch.  ctr
// (the phase counter, one word) must be zero when it starts.
// cands (optional) receives the lm_head phase's candidates for the sampler
// (ctas = step_plan_grid) and st->cand_ok says which were left.
cudaError_t step_launch(const StepPlan* plan, DecodeState* st, const float* rope, float eps,
                        float* part, uint32_t* ctr, int32_t* err, const LogitCands* cands, cudaStream_t s);

// ---------------------------------------------------------- prefill GEMM
// OUT[t*ldo + r] (+)= sum_k X[t*K + k] * W[r, k], t < n.
// Prefill matmul OUT[t][r] (+)= dot(X[t], W[r]).  With scratch of at least
// gemm_scratch_bytes(n, K) bytes (256-byte aligned) and K a multiple of 64 it
// runs on the tensor cores (tcgen05); otherwise on CUDA cores.
// x_split_ready (tensor-core path): the scratch already holds the fp16 split
// of this same X from the previous call (GEMMs that share their input).
// glu (tensor-core path, no split-K): OUT = silu(glu) * (X W^T), glu in OUT's
// layout (may be OUT itself): the SwiGLU of a gate projection fused.
cudaError_t gemm_launch(uint32_t type, const uint8_t* w, int64_t rows, int64_t K,
                        int64_t row_bytes, const float* X, int64_t n, float* out, int64_t ldo,
                        bool accumulate, void* scratch, size_t scratch_bytes, cudaStream_t s,
                        bool x_split_ready = false, const float* glu = nullptr);
// Whether gemm_launch takes the tensor-core path for these arguments.
bool gemm_uses_tc(uint32_t type, int64_t n, int64_t K, size_t scratch_bytes);
size_t gemm_scratch_bytes(int64_t n, int64_t K);
// tensor-core path (k_gemm_tc.cu)
size_t gemm_tc_scratch_bytes(int64_t n, int64_t K);
bool gemm_tc_supported(uint32_t type, int64_t K);
cudaError_t gemm_tc_launch(uint32_t type, const uint8_t* w, int64_t rows, int64_t K, int64_t row_bytes,
                           const float* X, int64_t n, float* out, int64_t ldo, bool accumulate,
                           void* scratch, size_t scratch_bytes, cudaStream_t s, bool x_split_ready,
                           const float* glu);
// Up to three matrices with the same input X (q, k and v) in one tensor-core
// launch (no split-K): OUT_i[t][r] = dot(X[t], W_i[r]).  Every matrix must
// pass gemm_uses_tc.
struct GemmGroupMat {
  uint32_t type;
  const uint8_t* w;
  int64_t rows, row_bytes;
  float* out;
  int64_t ldo;
};
cudaError_t gemm_tc_launch_group(const GemmGroupMat* mats, int nmat, int64_t K, const float* X, int64_t n,
                                 void* scratch, size_t scratch_bytes, cudaStream_t s, bool x_split_ready);
// The fp16 split of RMSNorm(X) * norm_w (rmsnorm_rows_launch's values) into
// the tensor-core scratch, for the GEMMs that follow with x_split_ready.
cudaError_t gemm_tc_split_norm(const float* X, const float* norm_w, float eps, int64_t n, int64_t K,
                               void* scratch, size_t scratch_bytes, cudaStream_t s);
// The fp16 split of silu(gate) * up (swiglu_launch's values) into the
// tensor-core scratch, for the down projection with x_split_ready.
cudaError_t gemm_tc_split_glu(const float* gate, const float* up, int64_t n, int64_t K, void* scratch,
                              size_t scratch_bytes, cudaStream_t s);

// -------------------------------------------------------------- others
cudaError_t dequant_launch(uint32_t type, const uint8_t* w, int64_t rows, int64_t cols,
                           int64_t row_bytes, float* out, cudaStream_t s);
// x[t] = dequant(embd row ids[t]); ids on device.  state (optional): take the
// single id from state->token and skip when inactive.  An id outside
// [0, n_rows) embeds as zeros and sets kErrBadToken in *err (optional).
cudaError_t embed_launch(uint32_t type, const uint8_t* embd, int64_t row_bytes, int64_t n_rows,
                         int32_t hidden, const int32_t* ids, int64_t n, float* x,
                         const DecodeState* state, int32_t* err, cudaStream_t s);
cudaError_t rmsnorm_rows_launch(const float* x, const float* w, int64_t n, int32_t dim, float eps,
                                float* out, cudaStream_t s);
// Batched decode: dst[b][0, n_cols) = src row b for every session b whose
// state is active (device arrays of n pointers).
cudaError_t commit_rows_launch(const float* src, int64_t n_cols, float* const* dst, DecodeState* const* states,
                               int32_t n, cudaStream_t s);
cudaError_t swiglu_launch(float* gate, const float* up, int64_t count, cudaStream_t s);

// Per token t (position pos0+t, or state->pos when state != null): RMSNorm
// each q and k head with its gain, RoPE both, write k and v into the cache.
struct QkvArgs {
  float* q;            // [n][n_heads*hd] in place
  const float* k;      // [n][n_kv*hd]
  const float* v;      // [n][n_kv*hd]
  const float* q_norm;
  const float* k_norm;
  const float* rope;   // [positions][hd/2 cos | hd/2 sin]
  float* kc;           // cache of this layer: [n_kv][max_seq][hd]
  float* vc;
  int64_t max_seq;
  int32_t n_heads, n_kv, hd;
  float eps;
  int64_t pos0;
  int64_t n;
  const DecodeState* state;
  int32_t kv_only;     // 1: only the k/v heads (the attention normalises and rotates q)
};
cudaError_t qkv_rope_launch(const QkvArgs& a, cudaStream_t s);

// One session of a batched decode step (attention over its own cache).
struct AttnBatchEntry {
  const DecodeState* state;  // position, active flag
  float* kc;                 // the session's K cache, layer 0 ([layers][n_kv][max_seq][hd])
  float* vc;
  int64_t max_seq;
  int32_t* err;              // the session's own error flags (a wait that gives up in its slice)
  int32_t stall;             // test hook: this session's layer-0 CTAs wait on a barrier nothing completes
};

struct AttnArgs {
  const float* q;      // [n][n_heads*hd] (decode with q_norm: raw projections)
  const float* kc;     // layer cache [n_kv][max_seq][hd]
  const float* vc;
  float* out;          // [n][n_heads*hd]
  int64_t max_seq;
  int32_t n_heads, n_kv, hd;
  int64_t pos0, n;     // prefill
  const DecodeState* state;  // decode: pos from state, n = 1
  int32_t* err;        // decode: optional error flags (bounded waits)
  // decode only, optional: fuse QK-norm + RoPE + K/V cache write of the new
  // token (q/k/v raw projections, k_new/v_new the token's k and v rows)
  const float* q_norm;
  const float* k_norm;
  const float* rope;
  const float* k_new;
  const float* v_new;
  float* kc_w;         // writable views of the caches
  float* vc_w;
  float eps;
  bool pdl;
  // batched decode (optional): nbatch sessions, blockIdx.z = session z, whose
  // q / k_new / v_new / out rows are row z of those arrays and whose cache is
  // layer `layer` of batch[z] (state, kc, vc, max_seq replace the fields above)
  const AttnBatchEntry* batch;
  int32_t nbatch, layer;
};
// Decode attention needs no scratch: the splits of a kv head form one
// thread-block cluster and merge in distributed shared memory.  Group sizes
// n_heads / n_kv of 1, 2, 4 or 8; head_dim 128; caches 16-byte aligned.
cudaError_t attn_decode_launch(const AttnArgs& a, cudaStream_t s);
cudaError_t attn_prefill_launch(const AttnArgs& a, cudaStream_t s);

// Sampler / argmax.  When state != null: decode-loop step (reads options,
// u = CounterUniform(seed, pos), writes state->token, appends to out_ids,
// updates done/active).  Otherwise samples with the explicit options into
// *token_out.
struct SampleArgs {
  const float* logits;
  int64_t n;
  float temperature;
  int32_t top_k;
  float top_p;
  float u;
  int32_t* token_out;
  DecodeState* state;
  int32_t* out_ids;
  int32_t* n_out;
  // decode loop: also gather the picked token's embedding row into x
  const uint8_t* embd;
  int64_t embd_row_bytes;
  uint32_t embd_type;
  int32_t hidden;
  float* x;
  bool pdl;
  // batched decode (optional): nbatch blocks, block b samples logits row b
  // (logits + b * n) for session b: states[b], out_ids_b[b], n_out_b[b], and
  // writes the embedding into x + b * hidden
  DecodeState* const* states;
  int32_t* const* out_ids_b;
  int32_t* const* n_out_b;
  int32_t nbatch;
  // decode loop (optional): the step kernel's candidates of the pending
  // logits, used when state->cand_ok says they fit the sampling options
  LogitCands cands;
};
cudaError_t sample_launch(const SampleArgs& a, cudaStream_t s);
// state->pos += 1 when active (end of a decode step).
cudaError_t advance_launch(DecodeState* st, cudaStream_t s);
// *st = v, ordered on the stream (the value travels as a kernel parameter, so
// the host may reuse its copy immediately).
cudaError_t state_set_launch(DecodeState* st, const DecodeState& v, cudaStream_t s);
// Number of active sessions among states[0, n) into *out (batched decode's early end).
cudaError_t count_active_launch(DecodeState* const* states, int32_t n, int32_t* out, cudaStream_t s);

}  // namespace rpgc
