// engine.cu -- host orchestration of the token loop and the rpgc C ABI.
//
// Mirrors the reference's token loop (src/qwen3.cc:119-355) and session
// model (src/engine.cc:383-448, src/kv_cache.h:35-82) with the compute on a
// B200: weights uploaded once as raw ggml blocks, one stream and one device
// KV cache per session, prefill through the batched kernels, and a decode
// loop that runs as one captured CUDA graph per step with its state (position,
// sampling options, stop status) in device memory.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <atomic>
#include <chrono>
#include <climits>
#include <condition_variable>
#include <deque>
#include <cstdlib>
#include <dlfcn.h>
#include <nccl.h>
#include <cstring>
#include <initializer_list>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/rpgc.h"
#include "gguf_host.h"
#include "kernels.h"

namespace rpgc {
namespace {

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

thread_local std::string g_last_error;

[[noreturn]] void fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  throw Error(code, buf);
}

#define CK(expr)                                                                      \
  do {                                                                                \
    const cudaError_t e_ = (expr);                                                    \
    if (e_ != cudaSuccess)                                                            \
      fail(e_ == cudaErrorMemoryAllocation ? RPGC_E_OOM : RPGC_E_CUDA, "%s: %s (%s:%d)", \
           #expr, cudaGetErrorString(e_), __FILE__, __LINE__);                        \
  } while (0)

struct DevMatrix {
  uint32_t type = 0;
  int64_t rows = 0, cols = 0, row_bytes = 0;
  const uint8_t* w = nullptr;
};

struct DevLayer {
  const float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  DevMatrix q, k, v, o, gate, up, down;
};

// ------------------------------------------------------------------ NCCL
// Loaded at first use (libnccl.so.2; a host that already uses NCCL, such as
// torch, has it mapped), so the library has no link-time NCCL dependency.
struct NcclApi {
  decltype(&ncclGetUniqueId) get_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

const NcclApi* nccl_api() {
  static NcclApi api;
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_id = reinterpret_cast<decltype(api.get_id)>(dlsym(h, "ncclGetUniqueId"));
    api.init_rank = reinterpret_cast<decltype(api.init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    ok = api.get_id && api.init_rank && api.destroy && api.all_reduce && api.all_gather && api.error_string;
  });
  return ok ? &api : nullptr;
}

struct BatchRequest;

// Gathers concurrent rpgc_generate calls on sessions of one model into
// batched decode steps (rpgc_model_set_batching).
struct Batcher {
  std::mutex mu;
  std::condition_variable cv;
  std::deque<BatchRequest*> pending;
  bool leading = false;  // a caller is gathering or running a batch
  int32_t max_batch = 0;  // 0: off
  int32_t window_us = 0;
  int64_t batches = 0, requests = 0;  // batches of two or more sessions run, and their requests
};

// Device buffers and captured step graphs of batched decode, kept on the
// model between batches and grown when a larger batch arrives: after the
// first batch of a size, a batch neither allocates nor frees device memory
// (cudaFree synchronises the whole device, which would stall every other
// session's stream).  One batch at a time per model uses them (mu is held
// across batch_decode).
struct BatchCache {
  std::mutex mu;
  int32_t cap = 0;  // sessions the buffers hold
  std::vector<void*> ptrs;
  float *x = nullptr, *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
  float *gate = nullptr, *up = nullptr, *logits = nullptr;
  void* scratch = nullptr;
  DecodeState** states = nullptr;
  int32_t** outs = nullptr;
  int32_t** nouts = nullptr;
  float** dst = nullptr;
  AttnBatchEntry* entries = nullptr;
  int32_t* n_active = nullptr;       // device: sessions still active (early end)
  int32_t* n_active_host = nullptr;  // pinned copy
  struct StepGraph {
    cudaGraphExec_t exec = nullptr;
    int64_t kernels = 0;
  };
  std::map<int32_t, StepGraph> graphs;  // batch size -> one captured step over these buffers
  // Frees everything (the device is current; no batch is running).
  void release() {
    for (auto& g : graphs) cudaGraphExecDestroy(g.second.exec);
    graphs.clear();
    for (void* p : ptrs) cudaFree(p);
    ptrs.clear();
    if (n_active_host) cudaFreeHost(n_active_host);
    n_active_host = nullptr;
    cap = 0;
  }
};

struct Model {
  int device = 0;
  rpgc_model_config c{};   // this rank's shapes (heads, kv heads, intermediate of its shard)
  rpgc_model_config cg{};  // the whole model
  int32_t tp_rank = 0, tp_world = 1;
  ncclComm_t comm = nullptr;  // tensor parallelism (tp_world > 1)
  uint8_t* blob = nullptr;
  int64_t weight_bytes = 0;
  DevMatrix embd, lm_head;
  const float* out_norm = nullptr;
  std::vector<DevLayer> layers;
  float* rope = nullptr;
  int64_t n_rope = 0;
  std::vector<int32_t> sessions;
  // end-of-sequence and <|im_end|> token ids (-1: none), the model-level stop
  // ids of the token-level engine (src/model.cc:187, src/engine.cc:451-454)
  int32_t eos_id = -1, im_end_id = -1;
  Batcher batcher;
  BatchCache bcache;
  ~Model() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    bcache.release();
    if (blob) cudaFree(blob);
    if (rope) cudaFree(rope);
    if (comm && nccl_api()) nccl_api()->destroy(comm);
    cudaSetDevice(prev);
  }
};


struct Session {
  int32_t model_id = 0;
  Model* m = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  int64_t max_seq = 0, len = 0, cap = 0;
  bool has_logits = false;
  float *kc = nullptr, *vc = nullptr;
  float *x = nullptr, *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
  float *gate = nullptr, *up = nullptr, *logits = nullptr;
  float* logits_part = nullptr;  // tensor parallelism: this rank's vocabulary slice
  int32_t *ids = nullptr, *gen_out = nullptr, *n_out = nullptr;
  void* gscratch = nullptr;  // prefill GEMM: split activations
  size_t gscratch_bytes = 0;
  DecodeState* st = nullptr;
  DecodeState* st_host = nullptr;  // pinned
  cudaGraphExec_t step_graph = nullptr;
  int64_t graph_kernels = 0;  // kernels in step_graph
  // persistent decode step (k_step.cu); null: per-launch kernels
  StepPlan* step_plan = nullptr;
  bool step_planned = false;
  float* step_part = nullptr;     // attention partials
  LogitCands cands{};             // the step kernel's lm_head candidates for the sampler
  uint32_t* step_ctr = nullptr;   // the step kernel's phase counter
  size_t step_ctr_bytes = 0;
  std::vector<void*> allocs;
  std::vector<void*> ipc_mapped;  // tensor parallelism: peers' step-kernel buffers mapped here
  std::mutex mu;

  template <typename T>
  T* alloc(size_t count) {
    void* p = nullptr;
    CK(cudaMalloc(&p, count * sizeof(T)));
    allocs.push_back(p);
    return static_cast<T*>(p);
  }
  ~Session() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    if (step_graph) cudaGraphExecDestroy(step_graph);
    for (void* p : ipc_mapped) cudaIpcCloseMemHandle(p);
    step_plan_free(step_plan);
    for (void* p : allocs) cudaFree(p);
    if (st_host) cudaFreeHost(st_host);
    if (stream) cudaStreamDestroy(stream);
    cudaSetDevice(prev);
  }
  size_t layer_cache_floats() const {
    return (size_t)m->c.n_kv_heads * max_seq * m->c.head_dim;
  }
};

std::mutex g_mu;
std::unordered_map<int32_t, std::unique_ptr<Model>> g_models;
std::unordered_map<int32_t, std::unique_ptr<Session>> g_sessions;
int32_t g_next_model = 1, g_next_session = 1;

Model* model_locked(int32_t h) {
  auto it = g_models.find(h);
  if (it == g_models.end()) fail(RPGC_E_STATE, "invalid model handle %d", h);
  return it->second.get();
}
Session* session_locked(int32_t h) {
  auto it = g_sessions.find(h);
  if (it == g_sessions.end()) fail(RPGC_E_STATE, "invalid session handle %d", h);
  return it->second.get();
}
Session* require_session(int32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  return session_locked(h);
}

struct DeviceGuard {
  int prev = 0;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    CK(cudaSetDevice(dev));
  }
  ~DeviceGuard() { cudaSetDevice(prev); }
};

int64_t row_bytes_of(uint32_t type, int64_t cols) {
  int64_t be, bb;
  if (!ggml_block(type, &be, &bb) || cols % be) return -1;
  return cols / be * bb;
}

bool kernel_type(uint32_t t) { return t == RPGC_F32 || t == RPGC_Q8_0 || t == RPGC_Q4_K || t == RPGC_Q6_K; }

// ------------------------------------------------------------------ upload
struct TensorRef {
  const rpgc_tensor* t = nullptr;
  size_t offset = 0;
};

// One uploaded piece of a tensor: all of it, a range of its rows, or a range
// of its columns (the same block range of every row, packed).
struct Piece {
  const rpgc_tensor* t = nullptr;
  int kind = 0;  // 0 whole, 1 rows [a, b), 2 columns [a, b)
  int64_t a = 0, b = 0;
  size_t offset = 0, bytes = 0;
};

// One host-to-device copy of the upload: `rows` rows of `width` bytes,
// `stride` apart in the source, packed at dst.
struct CopyJob {
  uint8_t* dst;
  const uint8_t* src;
  size_t width, stride, rows;
};

// Copies the pieces into the device blob through pinned staging memory: up to
// 8 host threads, each with two pinned buffers and its own stream, take the
// chunks round-robin; a thread fills one buffer from the source (page faults
// of a mapped file and the copy run in parallel across threads) while the
// other buffer's DMA runs.  Chunks are 1-8 MB (smaller models get smaller
// chunks, so every upload runs this path).
void upload_pieces(uint8_t* blob, const std::vector<Piece>& pieces, int device) {
  size_t total = 0;
  for (const Piece& pc : pieces) total += pc.bytes;
  const int hw = (int)std::max(1u, std::thread::hardware_concurrency());
  const int T = std::max(1, std::min(8, hw));
  size_t chunk = (total / (size_t)(4 * T) + 65535) & ~size_t(65535);
  chunk = std::min<size_t>(std::max<size_t>(chunk, 1u << 20), 8u << 20);
  std::vector<CopyJob> jobs;
  for (const Piece& pc : pieces) {
    const rpgc_tensor* t = pc.t;
    if (!t->data) fail(RPGC_E_ARG, "tensor %s has no data", t->name);
    const uint8_t* src = static_cast<const uint8_t*>(t->data);
    uint8_t* dst = blob + pc.offset;
    if (pc.kind == 2) {  // the same column range of every row
      const size_t rb = (size_t)row_bytes_of(t->type, t->dims[0]), w = (size_t)row_bytes_of(t->type, pc.b - pc.a);
      src += row_bytes_of(t->type, pc.a);
      const size_t rows = (size_t)t->dims[1], per = std::max<size_t>(1, chunk / w);
      for (size_t r = 0; r < rows; r += per)
        jobs.push_back(CopyJob{dst + r * w, src + r * rb, w, rb, std::min(per, rows - r)});
    } else {
      if (pc.kind == 1) src += pc.a * row_bytes_of(t->type, t->dims[0]);
      for (size_t o = 0; o < pc.bytes; o += chunk) {
        const size_t n = std::min(chunk, pc.bytes - o);
        jobs.push_back(CopyJob{dst + o, src + o, n, n, 1});
      }
    }
  }
  if (jobs.empty()) return;
  size_t buf_bytes = 0;
  for (const CopyJob& j : jobs) buf_bytes = std::max(buf_bytes, j.width * j.rows);
  const int nth = (int)std::min<size_t>((size_t)T, jobs.size());
  std::atomic<bool> failed{false};
  std::mutex emu;
  std::string err;
  auto note = [&](cudaError_t e, const char* what) {
    if (e == cudaSuccess) return false;
    std::lock_guard<std::mutex> lk(emu);
    if (err.empty()) err = std::string(what) + ": " + cudaGetErrorString(e);
    failed = true;
    return true;
  };
  auto worker = [&](int i) {
    if (note(cudaSetDevice(device), "cudaSetDevice")) return;
    cudaStream_t st = nullptr;
    uint8_t* buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool ok = !note(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
    for (int b = 0; ok && b < 2; ++b) {
      ok = !note(cudaHostAlloc(reinterpret_cast<void**>(&buf[b]), buf_bytes, cudaHostAllocDefault), "cudaHostAlloc");
      if (ok) ok = !note(cudaEventCreateWithFlags(&ev[b], cudaEventDisableTiming), "cudaEventCreate");
    }
    int k = 0;
    for (size_t j = (size_t)i; ok && !failed && j < jobs.size(); j += (size_t)nth, ++k) {
      const int b = k & 1;
      if (k >= 2 && note(cudaEventSynchronize(ev[b]), "upload copy")) break;  // the buffer's last copy is done
      const CopyJob& J = jobs[j];
      if (J.rows == 1 || J.stride == J.width) {
        std::memcpy(buf[b], J.src, J.width * J.rows);
      } else {
        for (size_t r = 0; r < J.rows; ++r) std::memcpy(buf[b] + r * J.width, J.src + r * J.stride, J.width);
      }
      if (note(cudaMemcpyAsync(J.dst, buf[b], J.width * J.rows, cudaMemcpyHostToDevice, st), "cudaMemcpyAsync"))
        break;
      if (note(cudaEventRecord(ev[b], st), "cudaEventRecord")) break;
    }
    if (st) note(cudaStreamSynchronize(st), "upload copy");
    for (int b = 0; b < 2; ++b) {
      if (ev[b]) cudaEventDestroy(ev[b]);
      if (buf[b]) cudaFreeHost(buf[b]);
    }
    if (st) cudaStreamDestroy(st);
  };
  std::vector<std::thread> th;
  for (int i = 1; i < nth; ++i) th.emplace_back(worker, i);
  worker(0);
  for (std::thread& t : th) t.join();
  if (failed) fail(RPGC_E_CUDA, "model upload: %s", err.c_str());
}

// Rank `rank`'s shard of a tensor-parallel model (world ranks): whole heads,
// kv heads, intermediate rows and vocabulary rows, an equal contiguous range
// per rank in rank order.
rpgc_tp_shard tp_shard_of(const rpgc_model_config& c, int32_t rank, int32_t world) {
  if (world < 1 || world > 64 || rank < 0 || rank >= world)
    fail(RPGC_E_ARG, "tensor-parallel rank %d of %d", rank, world);
  if (c.n_heads <= 0 || c.n_kv_heads <= 0 || c.intermediate <= 0 || c.vocab <= 0 || c.head_dim <= 0)
    fail(RPGC_E_ARG, "incomplete model config");
  if (world > 1 && (c.n_heads % world || c.n_kv_heads % world || c.intermediate % world || c.vocab % world))
    fail(RPGC_E_ARG, "heads %d, kv heads %d, intermediate %d and vocab %d must divide by %d ranks",
         c.n_heads, c.n_kv_heads, c.intermediate, c.vocab, world);
  rpgc_tp_shard t{};
  t.n_heads = c.n_heads / world;
  t.n_kv_heads = c.n_kv_heads / world;
  t.intermediate = c.intermediate / world;
  auto range = [&](int64_t per, int64_t* r) {
    r[0] = per * rank;
    r[1] = per * (rank + 1);
  };
  range((int64_t)t.n_heads * c.head_dim, t.q_rows);
  range((int64_t)t.n_kv_heads * c.head_dim, t.kv_rows);
  range(t.intermediate, t.ffn_rows);
  range(c.vocab / world, t.vocab_rows);
  range((int64_t)t.n_heads * c.head_dim, t.o_cols);
  range(t.intermediate, t.down_cols);
  return t;
}

// Uploads the model, or with world > 1 rank `rank`'s tensor-parallel shard:
// q/k/v/gate/up and the untied output split by rows (heads, intermediate
// rows, vocabulary), o and down by columns (the same block range of every
// row), everything else whole.
int32_t upload(int device, const rpgc_model_config& cfg, const rpgc_tensor* tensors, int n,
               int32_t rank = 0, int32_t world = 1, const void* nccl_id = nullptr) {
  const rpgc_model_config& c = cfg;
  if (c.n_layers <= 0 || c.hidden <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
      c.head_dim <= 0 || c.intermediate <= 0 || c.vocab <= 0)
    fail(RPGC_E_ARG, "incomplete model config: layers=%d hidden=%d heads=%d kv=%d head_dim=%d ffn=%d "
         "vocab=%d", c.n_layers, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim, c.intermediate,
         c.vocab);
  if (c.n_heads % c.n_kv_heads) fail(RPGC_E_ARG, "heads %d not a multiple of kv heads %d", c.n_heads, c.n_kv_heads);
  if (c.head_dim != 128) fail(RPGC_E_ARG, "head_dim %d unsupported (kernels take 128)", c.head_dim);
  {
    const int g = c.n_heads / c.n_kv_heads;
    if (!(g == 1 || g == 2 || g == 4 || g == 8))
      fail(RPGC_E_ARG, "GQA group %d unsupported (1, 2, 4 or 8)", g);
  }
  if (c.hidden % 256 || c.intermediate % 32) fail(RPGC_E_ARG, "hidden/intermediate not block aligned");
  const rpgc_tp_shard sh = tp_shard_of(c, rank, world);
  rpgc_model_config cl = c;  // this rank's shapes
  cl.n_heads = sh.n_heads;
  cl.n_kv_heads = sh.n_kv_heads;
  cl.intermediate = sh.intermediate;
  if (!gemv_supported(c.hidden, true) || !gemv_supported(cl.intermediate, false) ||
      !gemv_supported((int64_t)cl.n_heads * c.head_dim, false))
    fail(RPGC_E_ARG, "decode kernels need hidden, intermediate and heads*head_dim to be multiples of "
                     "128 within the decode kernel's limits");
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) fail(RPGC_E_ARG, "device %d out of range (%d devices)", device, ndev);

  std::unordered_map<std::string, const rpgc_tensor*> byname;
  for (int i = 0; i < n; ++i) {
    if (!tensors[i].name) fail(RPGC_E_ARG, "tensor %d has no name", i);
    byname[tensors[i].name] = &tensors[i];
  }
  auto find = [&](const std::string& nm) -> const rpgc_tensor* {
    auto it = byname.find(nm);
    return it == byname.end() ? nullptr : it->second;
  };
  auto require = [&](const std::string& nm) -> const rpgc_tensor* {
    const rpgc_tensor* t = find(nm);
    if (!t) fail(RPGC_E_ARG, "tensor %s missing", nm.c_str());
    return t;
  };
  auto check_matrix = [&](const rpgc_tensor* t, int64_t rows, int64_t cols) {
    if (t->n_dims != 2 || t->dims[1] != rows || t->dims[0] != cols)
      fail(RPGC_E_ARG, "tensor %s shape mismatch: want [%lld,%lld] (rows x cols)", t->name,
           (long long)rows, (long long)cols);
    if (!kernel_type(t->type)) fail(RPGC_E_ARG, "tensor %s type %u has no kernel", t->name, t->type);
    const int64_t rb = row_bytes_of(t->type, cols);
    if (rb < 0 || t->n_bytes < rb * rows) fail(RPGC_E_ARG, "tensor %s too short", t->name);
  };
  auto check_norm = [&](const rpgc_tensor* t, int64_t len) {
    if (t->n_dims != 1 || t->dims[0] != len) fail(RPGC_E_ARG, "norm %s length mismatch", t->name);
    if (t->type != RPGC_F32) fail(RPGC_E_ARG, "norm %s must be F32", t->name);
  };
  const int64_t H = c.hidden, F = c.intermediate, qd = (int64_t)c.n_heads * c.head_dim,
                kvd = (int64_t)c.n_kv_heads * c.head_dim;

  auto model = std::make_unique<Model>();
  model->device = device;
  model->c = cl;
  model->cg = c;
  model->tp_rank = rank;
  model->tp_world = world;
  std::vector<Piece> pieces;
  std::unordered_map<const rpgc_tensor*, size_t> piece_of;
  auto add = [&](const rpgc_tensor* t, int kind, int64_t a, int64_t b) {
    Piece pc;
    pc.t = t;
    pc.kind = kind;
    pc.a = a;
    pc.b = b;
    if (kind == 0) {
      pc.bytes = (size_t)t->n_bytes;
    } else {
      const int64_t rows = t->dims[1], cols = t->dims[0];
      pc.bytes = kind == 1 ? (size_t)((b - a) * row_bytes_of(t->type, cols))
                           : (size_t)(rows * row_bytes_of(t->type, b - a));
    }
    piece_of[t] = pieces.size();
    pieces.push_back(pc);
  };
  auto rows_of = [&](const rpgc_tensor* t, const int64_t* r) {  // this rank's row range
    add(t, world > 1 ? 1 : 0, r[0], r[1]);
  };
  auto cols_of = [&](const rpgc_tensor* t, const int64_t* k) {  // this rank's column range
    int64_t be = 0, bb = 0;
    if (!ggml_block(t->type, &be, &bb) || k[0] % be || k[1] % be)
      fail(RPGC_E_ARG, "tensor %s: the columns per rank (%lld) split a %lld-element block", t->name,
           (long long)(k[1] - k[0]), (long long)be);
    add(t, world > 1 ? 2 : 0, k[0], k[1]);
  };
  const rpgc_tensor* emb = require("token_embd.weight");
  check_matrix(emb, c.vocab, H);
  add(emb, 0, 0, 0);
  const rpgc_tensor* out = find("output.weight");
  if (out) {
    check_matrix(out, c.vocab, H);
    rows_of(out, sh.vocab_rows);
  }
  const rpgc_tensor* onorm = require("output_norm.weight");
  check_norm(onorm, H);
  add(onorm, 0, 0, 0);
  struct LT {
    const rpgc_tensor *an, *fn, *qn, *kn, *q, *k, *v, *o, *g, *u, *d;
  };
  std::vector<LT> lts(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    LT& t = lts[l];
    t.an = require(p + "attn_norm.weight");
    t.fn = require(p + "ffn_norm.weight");
    t.qn = require(p + "attn_q_norm.weight");
    t.kn = require(p + "attn_k_norm.weight");
    t.q = require(p + "attn_q.weight");
    t.k = require(p + "attn_k.weight");
    t.v = require(p + "attn_v.weight");
    t.o = require(p + "attn_output.weight");
    t.g = require(p + "ffn_gate.weight");
    t.u = require(p + "ffn_up.weight");
    t.d = require(p + "ffn_down.weight");
    check_norm(t.an, H);
    check_norm(t.fn, H);
    check_norm(t.qn, c.head_dim);
    check_norm(t.kn, c.head_dim);
    check_matrix(t.q, qd, H);
    check_matrix(t.k, kvd, H);
    check_matrix(t.v, kvd, H);
    check_matrix(t.o, H, qd);
    check_matrix(t.g, F, H);
    check_matrix(t.u, F, H);
    check_matrix(t.d, H, F);
    for (const rpgc_tensor* x : {t.an, t.fn, t.qn, t.kn}) add(x, 0, 0, 0);
    rows_of(t.q, sh.q_rows);
    rows_of(t.k, sh.kv_rows);
    rows_of(t.v, sh.kv_rows);
    cols_of(t.o, sh.o_cols);
    rows_of(t.g, sh.ffn_rows);
    rows_of(t.u, sh.ffn_rows);
    cols_of(t.d, sh.down_cols);
  }
  size_t total = 0;
  for (Piece& pc : pieces) {
    pc.offset = total;
    total += (pc.bytes + 255) & ~size_t(255);
  }
  DeviceGuard dg(device);
  if (world > 1) {
    const NcclApi* api = nccl_api();
    if (!api) fail(RPGC_E_STATE, "tensor parallelism needs libnccl.so.2");
    if (!nccl_id) fail(RPGC_E_ARG, "null NCCL id");
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    const ncclResult_t r = api->init_rank(&model->comm, world, id, rank);
    if (r != ncclSuccess) fail(RPGC_E_CUDA, "ncclCommInitRank: %s", api->error_string(r));
  }
  CK(cudaMalloc(&model->blob, total));
  upload_pieces(model->blob, pieces, device);
  model->weight_bytes = 0;
  for (const Piece& pc : pieces) model->weight_bytes += (int64_t)pc.bytes;
  auto mat = [&](const rpgc_tensor* t) {
    const Piece& pc = pieces[piece_of[t]];
    DevMatrix d;
    d.type = t->type;
    d.rows = pc.kind == 1 ? pc.b - pc.a : t->dims[1];
    d.cols = pc.kind == 2 ? pc.b - pc.a : t->dims[0];
    d.row_bytes = row_bytes_of(t->type, d.cols);
    d.w = model->blob + pc.offset;
    return d;
  };
  auto vec = [&](const rpgc_tensor* t) {
    return reinterpret_cast<const float*>(model->blob + pieces[piece_of[t]].offset);
  };
  model->embd = mat(emb);
  if (out) {
    model->lm_head = mat(out);
  } else {  // tied: this rank's vocabulary rows of the embedding table
    model->lm_head = model->embd;
    model->lm_head.rows = sh.vocab_rows[1] - sh.vocab_rows[0];
    model->lm_head.w = model->embd.w + sh.vocab_rows[0] * model->embd.row_bytes;
  }
  model->out_norm = vec(onorm);
  model->layers.resize(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    DevLayer& d = model->layers[l];
    const LT& t = lts[l];
    d.attn_norm = vec(t.an);
    d.ffn_norm = vec(t.fn);
    d.q_norm = vec(t.qn);
    d.k_norm = vec(t.kn);
    d.q = mat(t.q);
    d.k = mat(t.k);
    d.v = mat(t.v);
    d.o = mat(t.o);
    d.gate = mat(t.g);
    d.up = mat(t.u);
    d.down = mat(t.d);
  }
  // RoPE table: angles in double, rounded to float (src/model.cc:122-145).
  const int32_t half = c.head_dim / 2;
  int64_t np = c.max_pos > c.context_length ? c.context_length : c.max_pos;
  if (np <= 0) np = 1;
  model->n_rope = np;
  std::vector<float> rope((size_t)np * c.head_dim);
  std::vector<double> inv(half);
  for (int i = 0; i < half; ++i)
    inv[i] = 1.0 / std::pow((double)c.rope_theta, (double)(2 * i) / (double)c.head_dim);
  for (int64_t p = 0; p < np; ++p)
    for (int i = 0; i < half; ++i) {
      const double ang = (double)p * inv[i];
      rope[p * c.head_dim + i] = (float)std::cos(ang);
      rope[p * c.head_dim + half + i] = (float)std::sin(ang);
    }
  CK(cudaMalloc(&model->rope, rope.size() * sizeof(float)));
  CK(cudaMemcpy(model->rope, rope.data(), rope.size() * sizeof(float), cudaMemcpyHostToDevice));

  std::lock_guard<std::mutex> lk(g_mu);
  if (g_next_model <= 0) fail(RPGC_E_STATE, "model handles exhausted");
  const int32_t h = g_next_model++;
  g_models.emplace(h, std::move(model));
  return h;
}

// ------------------------------------------------------------ sessions
int32_t session_create(int32_t model, int32_t max_seq) {
  Model* m;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    m = model_locked(model);
  }
  if (max_seq <= 0 || max_seq > m->n_rope)
    fail(RPGC_E_ARG, "max_seq=%d must be in (0, %lld]", max_seq, (long long)m->n_rope);
  auto s = std::make_unique<Session>();
  s->model_id = model;
  s->m = m;
  s->device = m->device;
  s->max_seq = max_seq;
  const rpgc_model_config& c = m->c;
  DeviceGuard dg(m->device);
  CK(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
  const size_t cache = (size_t)c.n_layers * s->layer_cache_floats();
  s->kc = s->alloc<float>(cache);
  s->vc = s->alloc<float>(cache);
  CK(cudaMemsetAsync(s->kc, 0, cache * sizeof(float), s->stream));
  CK(cudaMemsetAsync(s->vc, 0, cache * sizeof(float), s->stream));
  s->cap = std::min<int64_t>(512, max_seq);
  const int64_t H = c.hidden, F = c.intermediate, qd = (int64_t)c.n_heads * c.head_dim,
                kvd = (int64_t)c.n_kv_heads * c.head_dim;
  s->x = s->alloc<float>(s->cap * H);
  s->h = s->alloc<float>(s->cap * H);
  s->q = s->alloc<float>(s->cap * qd);
  s->k = s->alloc<float>(s->cap * kvd);
  s->v = s->alloc<float>(s->cap * kvd);
  s->attn = s->alloc<float>(s->cap * qd);
  s->gate = s->alloc<float>(s->cap * F);
  s->up = s->alloc<float>(s->cap * F);
  s->logits = s->alloc<float>(c.vocab);
  if (m->tp_world > 1) s->logits_part = s->alloc<float>(c.vocab / m->tp_world);
  {
    int64_t kmax = H > qd ? H : qd;
    kmax = kmax > F ? kmax : F;
    s->gscratch_bytes = gemm_scratch_bytes(s->cap, kmax);
    s->gscratch = s->alloc<uint8_t>(s->gscratch_bytes);
  }
  s->ids = s->alloc<int32_t>(s->cap);
  s->gen_out = s->alloc<int32_t>(max_seq + 1);
  s->n_out = s->alloc<int32_t>(1);
  s->st = s->alloc<DecodeState>(1);
  CK(cudaMallocHost(&s->st_host, sizeof(DecodeState)));
  std::memset(s->st_host, 0, sizeof(DecodeState));
  CK(cudaMemsetAsync(s->st, 0, sizeof(DecodeState), s->stream));
  CK(cudaStreamSynchronize(s->stream));
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_next_session <= 0) fail(RPGC_E_STATE, "session handles exhausted");
  const int32_t h = g_next_session++;
  m->sessions.push_back(h);
  g_sessions.emplace(h, std::move(s));
  return h;
}

// ------------------------------------------------------------- forward
void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(e == cudaErrorInvalidValue ? RPGC_E_ARG : RPGC_E_CUDA, "%s: %s", what,
                             cudaGetErrorString(e));
}

GemvSeg seg_of(const DevMatrix& d, float* out, int32_t mode) {
  GemvSeg s;
  s.w = d.w;
  s.out = out;
  s.rows = d.rows;
  s.row_bytes = d.row_bytes;
  s.type = d.type;
  s.mode = mode;
  return s;
}

// ------------------------------------------------ tensor-parallel collectives
// Sum of every rank's partial `buf` (count floats) in place.
void tp_all_reduce(Session* s, float* buf, size_t count) {
  const Model* m = s->m;
  if (m->tp_world <= 1) return;
  const ncclResult_t r = nccl_api()->all_reduce(buf, buf, count, ncclFloat, ncclSum, m->comm, s->stream);
  if (r != ncclSuccess) fail(RPGC_E_CUDA, "ncclAllReduce: %s", nccl_api()->error_string(r));
}
// The ranks' vocabulary slices of the logits (logits_part) into s->logits.
void tp_gather_logits(Session* s) {
  const Model* m = s->m;
  const ncclResult_t r = nccl_api()->all_gather(s->logits_part, s->logits, (size_t)m->c.vocab / m->tp_world,
                                                ncclFloat, m->comm, s->stream);
  if (r != ncclSuccess) fail(RPGC_E_CUDA, "ncclAllGather: %s", nccl_api()->error_string(r));
}
// Row-split matmuls (o, down) under tensor parallelism: rank 0 adds its
// partial to the residual, the others store theirs, and the all-reduce sums
// them into the new residual on every rank.
int32_t residual_mode(const Session* s) { return s->m->tp_rank == 0 ? kAdd : kStore; }
float* lm_head_out(Session* s) { return s->m->tp_world > 1 ? s->logits_part : s->logits; }

// Bytes of the next launch's rows each CTA prefetches into L2 per matrix.
constexpr int32_t kPrefetchBytes = 64 * 1024;

// L2 prefetch of the matrices of the next matrix-vector launch of the step.
void prefetch_of(GemvArgs* g, std::initializer_list<const DevMatrix*> next) {
  g->npf = 0;
  for (const DevMatrix* d : next) {
    GemvPrefetch& f = g->pf[g->npf++];
    f.w = d->w;
    f.rows = d->rows;
    f.row_bytes = d->row_bytes;
  }
  g->pf_bytes = kPrefetchBytes;
}

// Common GEMV arguments of a decode step (the session's active flag and
// error flags).
GemvArgs step_gemv(Session* s, const float* x, int32_t K, const float* norm_w) {
  GemvArgs g{};
  g.K = K;
  g.x = x;
  g.norm_w = norm_w;
  g.eps = s->m->c.rms_eps;
  g.active = &s->st->active;
  g.err = &s->st->error;
  return g;
}

// Whether the persistent decode-step kernel is enabled (RPGC_STEP_KERNEL=0
// selects the per-launch kernels, for comparison).
bool step_kernel_enabled() {
  const char* e = std::getenv("RPGC_STEP_KERNEL");
  return !(e && e[0] == '0' && e[1] == 0);
}

// Every rank's address of two device allocations of every rank (this rank's
// own at its index): the IPC handles all-gathered over the model's
// communicator, the peers' mapped with peer access.  The mappings are closed
// with the session.
void tp_map_peers(Session* s, void* a_own, void* b_own, std::vector<void*>* a_all, std::vector<void*>* b_all) {
  const Model* m = s->m;
  const int W = m->tp_world, R = m->tp_rank;
  cudaIpcMemHandle_t own[2];
  CK(cudaIpcGetMemHandle(&own[0], a_own));
  CK(cudaIpcGetMemHandle(&own[1], b_own));
  const size_t hb = sizeof(own);
  std::vector<cudaIpcMemHandle_t> all((size_t)2 * W);
  char* dev = nullptr;
  CK(cudaMalloc(&dev, hb * (W + 1)));
  try {
    CK(cudaMemcpyAsync(dev + hb * W, own, hb, cudaMemcpyHostToDevice, s->stream));
    const ncclResult_t r = nccl_api()->all_gather(dev + hb * W, dev, hb, ncclChar, m->comm, s->stream);
    if (r != ncclSuccess) fail(RPGC_E_CUDA, "ncclAllGather: %s", nccl_api()->error_string(r));
    CK(cudaMemcpyAsync(all.data(), dev, hb * W, cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
  } catch (...) {
    cudaFree(dev);
    throw;
  }
  cudaFree(dev);
  a_all->assign(W, nullptr);
  b_all->assign(W, nullptr);
  for (int r = 0; r < W; ++r) {
    if (r == R) {
      (*a_all)[r] = a_own;
      (*b_all)[r] = b_own;
      continue;
    }
    for (int k = 0; k < 2; ++k) {
      void* p = nullptr;
      CK(cudaIpcOpenMemHandle(&p, all[(size_t)2 * r + k], cudaIpcMemLazyEnablePeerAccess));
      s->ipc_mapped.push_back(p);
      (k ? *b_all : *a_all)[r] = p;
    }
  }
}

// Plans the persistent decode step of a session once (device allocations:
// call outside graph capture).  Leaves step_plan null when the model's block
// types or shapes are outside the step kernel, or it is disabled.  Under
// tensor parallelism every rank plans at the same call (the peers' buffers
// are exchanged over the communicator); the o and down projections leave
// partial rows in every rank's inbox, the phase after each sums them onto
// the residual, and the vocabulary-split lm_head writes its rows into every
// rank's logits, so the decode step runs no collective call.
void ensure_step_plan(Session* s) {
  if (s->step_planned) return;
  s->step_planned = true;
  if (!step_kernel_enabled()) return;
  const Model* m = s->m;
  const bool tp = m->tp_world > 1;
  const rpgc_model_config& c = m->c;
  const size_t lc = s->layer_cache_floats();
  const int32_t qd = c.n_heads * c.head_dim;
  s->step_ctr_bytes = sizeof(uint32_t);
  s->step_ctr = s->alloc<uint32_t>(1);
  std::vector<StepPhaseIn> ph;
  auto gemv_phase = [&](const float* x, int32_t K, const float* norm) {
    StepPhaseIn p;
    std::memset(&p, 0, sizeof(p));
    p.kind = 0;
    p.g.x = x;
    p.g.K = K;
    p.g.norm_w = norm;
    return p;
  };
  // under tensor parallelism the row-split projections store partial rows
  // (exchanged), otherwise they add into the residual
  const int32_t res_mode = tp ? kStore : kAdd;
  for (int l = 0; l < c.n_layers; ++l) {
    const DevLayer& L = m->layers[l];
    StepPhaseIn q = gemv_phase(s->x, c.hidden, L.attn_norm);
    q.g.seg[0] = seg_of(L.q, s->q, kStore);
    q.g.seg[1] = seg_of(L.k, s->k, kStore);
    q.g.seg[2] = seg_of(L.v, s->v, kStore);
    q.g.nseg = 3;
    q.x_sum = tp && l > 0;
    ph.push_back(q);
    StepPhaseIn a;
    std::memset(&a, 0, sizeof(a));
    a.kind = 1;
    a.a.q = s->q;
    a.a.k_new = s->k;
    a.a.v_new = s->v;
    a.a.q_norm = L.q_norm;
    a.a.k_norm = L.k_norm;
    a.a.kc = s->kc + l * lc;
    a.a.vc = s->vc + l * lc;
    a.a.out = s->attn;
    ph.push_back(a);
    StepPhaseIn o = gemv_phase(s->attn, qd, nullptr);
    o.g.seg[0] = seg_of(L.o, s->x, res_mode);
    o.g.nseg = 1;
    o.xchg = tp ? 1 : 0;
    ph.push_back(o);
    StepPhaseIn f = gemv_phase(s->x, c.hidden, L.ffn_norm);
    f.g.seg[0] = seg_of(L.gate, s->gate, kSwiGLU);
    f.g.seg[1] = seg_of(L.up, s->gate, kStore);
    f.g.nseg = 2;
    f.x_sum = tp;
    ph.push_back(f);
    StepPhaseIn d = gemv_phase(s->gate, c.intermediate, nullptr);
    d.g.seg[0] = seg_of(L.down, s->x, res_mode);
    d.g.nseg = 1;
    d.xchg = tp ? 1 : 0;
    ph.push_back(d);
  }
  StepPhaseIn h = gemv_phase(s->x, c.hidden, m->out_norm);
  h.g.seg[0] = seg_of(m->lm_head, tp ? s->logits_part : s->logits, kStore);
  h.g.nseg = 1;
  h.cand = tp ? 0 : 1;
  h.x_sum = tp;
  h.xchg = tp ? 2 : 0;
  ph.push_back(h);
  StepTp spec{m->tp_rank, m->tp_world, c.hidden, (int64_t)m->tp_rank * m->lm_head.rows};
  StepPlan* plan = nullptr;
  if (step_plan_create(ph.data(), (int)ph.size(), c.n_heads, c.n_kv_heads, s->max_seq, s->device, &plan,
                       tp ? &spec : nullptr) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  if (tp) {
    // every rank reaches this call (the same forward or generate on every
    // rank); a rank whose plan failed above fails the exchange's peers too
    std::vector<void*> arenas, outs;
    try {
      tp_map_peers(s, step_plan_tp_arena(plan), s->logits, &arenas, &outs);
    } catch (...) {
      step_plan_free(plan);
      throw;
    }
    std::vector<float*> outf(outs.size());
    for (size_t r = 0; r < outs.size(); ++r) outf[r] = static_cast<float*>(outs[r]);
    if (step_plan_tp_bind(plan, arenas.data(), outf.data()) != cudaSuccess) {
      step_plan_free(plan);
      fail(RPGC_E_CUDA, "binding the tensor-parallel decode step failed");
    }
    s->step_plan = plan;
    s->step_part = s->alloc<float>(step_part_floats(plan));
    return;  // candidates: the sampler sweeps the gathered logits
  }
  s->step_plan = plan;
  s->step_part = s->alloc<float>(step_part_floats(plan));
  const int ctas = step_plan_grid(plan);
  s->cands.ctas = ctas;
  s->cands.val = s->alloc<float>((size_t)ctas * kCandK);
  s->cands.idx = s->alloc<int32_t>((size_t)ctas * kCandK);
  s->cands.max_val = s->alloc<float>((size_t)ctas);
  s->cands.max_idx = s->alloc<int32_t>((size_t)ctas);
}

// Transformer layers + lm_head of one decode step for the token whose
// embedding is already in s->x, at position st->pos.  Every kernel honours
// st->active and is launched as a programmatic dependent of the previous one,
// so each GEMV's weight streaming starts while its predecessor finishes.
void launch_layers_step(Session* s) {
  if (s->step_plan) {
    CK(cudaMemsetAsync(s->step_ctr, 0, s->step_ctr_bytes, s->stream));
    check(step_launch(s->step_plan, s->st, s->m->rope, s->m->c.rms_eps, s->step_part, s->step_ctr,
                      &s->st->error, &s->cands, s->stream),
          "decode step");
    return;
  }
  const Model* m = s->m;
  const rpgc_model_config& c = m->c;
  cudaStream_t cs = s->stream;
  const size_t lc = s->layer_cache_floats();
  const int32_t qd = c.n_heads * c.head_dim;
  for (int l = 0; l < c.n_layers; ++l) {
    const DevLayer& L = m->layers[l];
    GemvArgs g = step_gemv(s, s->x, c.hidden, L.attn_norm);
    g.seg[0] = seg_of(L.q, s->q, kStore);
    g.seg[1] = seg_of(L.k, s->k, kStore);
    g.seg[2] = seg_of(L.v, s->v, kStore);
    g.nseg = 3;
    prefetch_of(&g, {&L.o});
    check(gemv_launch(g, cs, true), "gemv qkv");
    AttnArgs aa{};
    aa.q = s->q;
    aa.kc = s->kc + l * lc;
    aa.vc = s->vc + l * lc;
    aa.kc_w = s->kc + l * lc;
    aa.vc_w = s->vc + l * lc;
    aa.k_new = s->k;
    aa.v_new = s->v;
    aa.q_norm = L.q_norm;
    aa.k_norm = L.k_norm;
    aa.rope = m->rope;
    aa.eps = c.rms_eps;
    aa.out = s->attn;
    aa.max_seq = s->max_seq;
    aa.n_heads = c.n_heads;
    aa.n_kv = c.n_kv_heads;
    aa.hd = c.head_dim;
    aa.n = 1;
    aa.state = s->st;
    aa.err = &s->st->error;
    aa.pdl = true;
    check(attn_decode_launch(aa, cs), "attn decode");
    GemvArgs go = step_gemv(s, s->attn, qd, nullptr);
    go.seg[0] = seg_of(L.o, s->x, residual_mode(s));
    go.nseg = 1;
    prefetch_of(&go, {&L.gate, &L.up});
    check(gemv_launch(go, cs, true), "gemv o");
    tp_all_reduce(s, s->x, c.hidden);
    GemvArgs gf = step_gemv(s, s->x, c.hidden, L.ffn_norm);
    gf.seg[0] = seg_of(L.gate, s->gate, kSwiGLU);
    gf.seg[1] = seg_of(L.up, s->gate, kStore);
    gf.nseg = 2;
    prefetch_of(&gf, {&L.down});
    check(gemv_launch(gf, cs, true), "gemv gate/up");
    GemvArgs gd = step_gemv(s, s->gate, c.intermediate, nullptr);
    gd.seg[0] = seg_of(L.down, s->x, residual_mode(s));
    gd.nseg = 1;
    if (l + 1 < c.n_layers) {
      const DevLayer& N = m->layers[l + 1];
      prefetch_of(&gd, {&N.q, &N.k, &N.v});
    } else {
      prefetch_of(&gd, {&m->lm_head});
    }
    check(gemv_launch(gd, cs, true), "gemv down");
    tp_all_reduce(s, s->x, c.hidden);
  }
  GemvArgs gl = step_gemv(s, s->x, c.hidden, m->out_norm);
  gl.seg[0] = seg_of(m->lm_head, lm_head_out(s), kStore);
  gl.nseg = 1;
  prefetch_of(&gl, {&m->layers[0].q, &m->layers[0].k, &m->layers[0].v});  // the next step
  check(gemv_launch(gl, cs, true), "gemv lm_head");
  if (m->tp_world > 1) tp_gather_logits(s);
}

// One decode step for ids[0] at st->pos (the host set the state).
void launch_step(Session* s) {
  const Model* m = s->m;
  check(embed_launch(m->embd.type, m->embd.w, m->embd.row_bytes, m->embd.rows, m->c.hidden, s->ids, 1,
                     s->x, nullptr, &s->st->error, s->stream),
        "embed");
  launch_layers_step(s);
}

// Prefill of nc tokens (ids already in s->ids) at positions [pos0, pos0+nc).
void launch_prefill(Session* s, int64_t nc, int64_t pos0) {
  const Model* m = s->m;
  const rpgc_model_config& c = m->c;
  cudaStream_t cs = s->stream;
  const int64_t H = c.hidden, F = c.intermediate, qd = (int64_t)c.n_heads * c.head_dim,
                kvd = (int64_t)c.n_kv_heads * c.head_dim;
  check(embed_launch(m->embd.type, m->embd.w, m->embd.row_bytes, m->embd.rows, c.hidden, s->ids, nc,
                     s->x, nullptr, &s->st->error, cs),
        "embed");
  const size_t lc = s->layer_cache_floats();
  for (int l = 0; l < c.n_layers; ++l) {
    const DevLayer& L = m->layers[l];
    // q, k and v share their input: one fp16 split of the normalised rows
    // (the RMSNorm fused into it) and one launch serve the three tensor-core
    // GEMMs
    const bool tq = gemm_uses_tc(L.q.type, nc, H, s->gscratch_bytes);
    const bool tk = gemm_uses_tc(L.k.type, nc, H, s->gscratch_bytes);
    const bool tv = gemm_uses_tc(L.v.type, nc, H, s->gscratch_bytes);
    if (tq && tk && tv) {  // one launch over the three matrices' tiles
      const GemmGroupMat qkv[3] = {{L.q.type, L.q.w, L.q.rows, L.q.row_bytes, s->q, qd},
                                   {L.k.type, L.k.w, L.k.rows, L.k.row_bytes, s->k, kvd},
                                   {L.v.type, L.v.w, L.v.rows, L.v.row_bytes, s->v, kvd}};
      check(gemm_tc_split_norm(s->x, L.attn_norm, c.rms_eps, nc, H, s->gscratch, s->gscratch_bytes, cs), "norm split");
      check(gemm_tc_launch_group(qkv, 3, H, nullptr, nc, s->gscratch, s->gscratch_bytes, cs, true), "gemm qkv");
    } else {
      check(rmsnorm_rows_launch(s->x, L.attn_norm, nc, c.hidden, c.rms_eps, s->h, cs), "rmsnorm");
      check(gemm_launch(L.q.type, L.q.w, L.q.rows, H, L.q.row_bytes, s->h, nc, s->q, qd, false, s->gscratch, s->gscratch_bytes, cs), "gemm q");
      check(gemm_launch(L.k.type, L.k.w, L.k.rows, H, L.k.row_bytes, s->h, nc, s->k, kvd, false, s->gscratch, s->gscratch_bytes, cs, tq && tk), "gemm k");
      check(gemm_launch(L.v.type, L.v.w, L.v.rows, H, L.v.row_bytes, s->h, nc, s->v, kvd, false, s->gscratch, s->gscratch_bytes, cs, (tq || tk) && tv && tk), "gemm v");
    }
    QkvArgs qa{};
    qa.q = s->q;
    qa.k = s->k;
    qa.v = s->v;
    qa.q_norm = L.q_norm;
    qa.k_norm = L.k_norm;
    qa.rope = m->rope;
    qa.kc = s->kc + l * lc;
    qa.vc = s->vc + l * lc;
    qa.max_seq = s->max_seq;
    qa.n_heads = c.n_heads;
    qa.n_kv = c.n_kv_heads;
    qa.hd = c.head_dim;
    qa.eps = c.rms_eps;
    qa.pos0 = pos0;
    qa.n = nc;
    qa.kv_only = 1;  // the attention kernel normalises and rotates q as it loads it
    check(qkv_rope_launch(qa, cs), "qkv rope");
    AttnArgs aa{};
    aa.q = s->q;
    aa.kc = s->kc + l * lc;
    aa.vc = s->vc + l * lc;
    aa.out = s->attn;
    aa.max_seq = s->max_seq;
    aa.n_heads = c.n_heads;
    aa.n_kv = c.n_kv_heads;
    aa.hd = c.head_dim;
    aa.pos0 = pos0;
    aa.n = nc;
    aa.q_norm = L.q_norm;
    aa.rope = m->rope;
    aa.eps = c.rms_eps;
    check(attn_prefill_launch(aa, cs), "attn prefill");
    check(gemm_launch(L.o.type, L.o.w, L.o.rows, qd, L.o.row_bytes, s->attn, nc, s->x, H, m->tp_rank == 0, s->gscratch, s->gscratch_bytes, cs), "gemm o");
    tp_all_reduce(s, s->x, (size_t)nc * H);
    if (gemm_uses_tc(L.gate.type, nc, H, s->gscratch_bytes) && gemm_uses_tc(L.up.type, nc, H, s->gscratch_bytes) &&
        gemm_uses_tc(L.down.type, nc, F, s->gscratch_bytes)) {
      // the normalised rows only as their fp16 split (gate and up share it);
      // SwiGLU inside the split of the down projection's input
      check(gemm_tc_split_norm(s->x, L.ffn_norm, c.rms_eps, nc, H, s->gscratch, s->gscratch_bytes, cs), "norm split");
      check(gemm_launch(L.gate.type, L.gate.w, L.gate.rows, H, L.gate.row_bytes, nullptr, nc, s->gate, F, false, s->gscratch, s->gscratch_bytes, cs, true), "gemm gate");
      check(gemm_launch(L.up.type, L.up.w, L.up.rows, H, L.up.row_bytes, nullptr, nc, s->up, F, false, s->gscratch, s->gscratch_bytes, cs, true), "gemm up");
      check(gemm_tc_split_glu(s->gate, s->up, nc, F, s->gscratch, s->gscratch_bytes, cs), "glu split");
      check(gemm_launch(L.down.type, L.down.w, L.down.rows, F, L.down.row_bytes, nullptr, nc, s->x, H, m->tp_rank == 0, s->gscratch, s->gscratch_bytes, cs, true), "gemm down");
    } else {
      check(rmsnorm_rows_launch(s->x, L.ffn_norm, nc, c.hidden, c.rms_eps, s->h, cs), "rmsnorm");
      check(gemm_launch(L.gate.type, L.gate.w, L.gate.rows, H, L.gate.row_bytes, s->h, nc, s->gate, F, false, s->gscratch, s->gscratch_bytes, cs), "gemm gate");
      check(gemm_launch(L.up.type, L.up.w, L.up.rows, H, L.up.row_bytes, s->h, nc, s->up, F, false, s->gscratch, s->gscratch_bytes, cs), "gemm up");
      check(swiglu_launch(s->gate, s->up, nc * F, cs), "swiglu");
      check(gemm_launch(L.down.type, L.down.w, L.down.rows, F, L.down.row_bytes, s->gate, nc, s->x, H, m->tp_rank == 0, s->gscratch, s->gscratch_bytes, cs), "gemm down");
    }
    tp_all_reduce(s, s->x, (size_t)nc * H);
  }
}

void set_state_for_forward(Session* s) {
  DecodeState h;
  std::memset(&h, 0, sizeof(h));
  h.pos = (int32_t)s->len;
  h.active = 1;
  check(state_set_launch(s->st, h, s->stream), "state");
}

// Shared body of rpgc_forward / rpgc_forward_device.
void forward(Session* s, const int32_t* ids, bool ids_on_device, int64_t n, float* last,
             float* all) {
  const Model* m = s->m;
  const rpgc_model_config& c = m->c;
  if (n <= 0) fail(RPGC_E_ARG, "empty prompt");
  if (s->len + n > m->n_rope)
    fail(RPGC_E_ARG, "position %lld exceeds the RoPE table (%lld positions)",
         (long long)(s->len + n), (long long)m->n_rope);
  if (s->len + n > s->max_seq)
    fail(RPGC_E_CONTEXT_FULL, "position %lld exceeds the KV cache capacity %lld",
         (long long)(s->len + n), (long long)s->max_seq);
  if (!ids_on_device)
    for (int64_t t = 0; t < n; ++t)
      if (ids[t] < 0 || ids[t] >= c.vocab)
        fail(RPGC_E_ARG, "token %lld id %d out of range (vocab %d)", (long long)t, ids[t], c.vocab);
  DeviceGuard dg(s->device);
  s->has_logits = false;
  float* all_dev = nullptr;
  float* all_part = nullptr;  // tensor parallelism: [world][rows][vocab / world] gathered slices
  const int64_t vl = c.vocab / m->tp_world;
  if (all) CK(cudaMalloc(&all_dev, (size_t)s->cap * c.vocab * sizeof(float)));
  if (all && m->tp_world > 1) CK(cudaMalloc(&all_part, (size_t)(m->tp_world + 1) * s->cap * vl * sizeof(float)));
  try {
    for (int64_t t0 = 0; t0 < n; t0 += s->cap) {
      const int64_t nc = std::min<int64_t>(s->cap, n - t0);
      CK(cudaMemcpyAsync(s->ids, ids + t0, nc * sizeof(int32_t),
                         ids_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                         s->stream));
      if (nc == 1 && !all) {
        set_state_for_forward(s);
        ensure_step_plan(s);
        launch_step(s);
      } else {
        launch_prefill(s, nc, s->len);
        if (all) {
          check(rmsnorm_rows_launch(s->x, m->out_norm, nc, c.hidden, c.rms_eps, s->h, s->stream),
                "rmsnorm");
          if (m->tp_world > 1) {  // this rank's slice, gathered, then interleaved by rows
            float* mine = all_part + (size_t)m->tp_world * s->cap * vl;
            check(gemm_launch(m->lm_head.type, m->lm_head.w, m->lm_head.rows, c.hidden,
                              m->lm_head.row_bytes, s->h, nc, mine, vl, false, s->gscratch,
                              s->gscratch_bytes, s->stream),
                  "gemm lm_head");
            const ncclResult_t r = nccl_api()->all_gather(mine, all_part, (size_t)nc * vl, ncclFloat,
                                                          m->comm, s->stream);
            if (r != ncclSuccess) fail(RPGC_E_CUDA, "ncclAllGather: %s", nccl_api()->error_string(r));
            check(gather_vocab_launch(all_part, m->tp_world, nc, vl, all_dev, s->stream), "gather logits");
          } else {
            check(gemm_launch(m->lm_head.type, m->lm_head.w, m->lm_head.rows, c.hidden,
                              m->lm_head.row_bytes, s->h, nc, all_dev, c.vocab, false, s->gscratch,
                              s->gscratch_bytes, s->stream),
                  "gemm lm_head");
          }
          CK(cudaMemcpyAsync(all + t0 * c.vocab, all_dev, (size_t)nc * c.vocab * sizeof(float),
                             cudaMemcpyDeviceToHost, s->stream));
        }
        if (t0 + nc == n) {  // last row -> pending logits
          GemvArgs gl{};
          gl.seg[0] = seg_of(m->lm_head, lm_head_out(s), kStore);
          gl.nseg = 1;
          gl.K = c.hidden;
          gl.x = s->x + (nc - 1) * c.hidden;
          gl.norm_w = m->out_norm;
          gl.eps = c.rms_eps;
          check(gemv_launch(gl, s->stream, false), "gemv lm_head");
          if (m->tp_world > 1) tp_gather_logits(s);
        }
      }
      s->len += nc;
    }
    if (last)
      CK(cudaMemcpyAsync(last, s->logits, c.vocab * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
    if (last || all || !ids_on_device) CK(cudaStreamSynchronize(s->stream));
  } catch (...) {
    if (all_dev) cudaFree(all_dev);
    if (all_part) cudaFree(all_part);
    throw;
  }
  if (all_dev) cudaFree(all_dev);
  if (all_part) cudaFree(all_part);
  s->has_logits = true;
}

// Kernel launches enqueued by this thread while it captures a graph are
// counted into the graph, not as launches.
thread_local int64_t* t_capture_count = nullptr;
std::atomic<int64_t> g_launches{0};

void capture_step_graph(Session* s) {
  if (s->step_graph) return;
  ensure_step_plan(s);
  cudaGraph_t g = nullptr;
  int64_t nk = 0;
  CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  t_capture_count = &nk;
  try {
    const Model* m = s->m;
    SampleArgs sa{};
    sa.logits = s->logits;
    sa.n = m->c.vocab;
    sa.state = s->st;
    sa.out_ids = s->gen_out;
    sa.n_out = s->n_out;
    sa.embd = m->embd.w;
    sa.embd_row_bytes = m->embd.row_bytes;
    sa.embd_type = m->embd.type;
    sa.hidden = m->c.hidden;
    sa.x = s->x;
    sa.pdl = true;
    sa.cands = s->cands;  // ctas 0 without a step plan: the full sweep
    check(sample_launch(sa, s->stream), "sample");
    launch_layers_step(s);
  } catch (...) {
    t_capture_count = nullptr;
    cudaStreamEndCapture(s->stream, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  t_capture_count = nullptr;
  CK(cudaStreamEndCapture(s->stream, &g));
  const cudaError_t e = cudaGraphInstantiate(&s->step_graph, g, 0);
  cudaGraphDestroy(g);
  CK(e);
  s->graph_kernels = nk;
}

// Shared body of rpgc_generate / rpgc_generate_device.  Returns the number of
// steps launched.
int64_t generate(Session* s, const rpgc_gen_opts& o, bool sync_host) {
  const rpgc_model_config& c = s->m->c;
  if (!s->has_logits) fail(RPGC_E_STATE, "no pending logits: call rpgc_forward first");
  if (o.max_tokens <= 0) fail(RPGC_E_ARG, "max_tokens must be positive, got %d", o.max_tokens);
  if (o.n_stop < 0 || o.n_stop > RPGC_MAX_STOP) fail(RPGC_E_ARG, "at most %d stop ids", RPGC_MAX_STOP);
  if (o.n_stop > 0 && !o.stop_ids) fail(RPGC_E_ARG, "stop_ids is NULL");
  const int64_t room = s->max_seq - s->len;
  if (room <= 0)
    fail(RPGC_E_CONTEXT_FULL, "context full (%lld positions)", (long long)s->max_seq);
  const int64_t steps = std::min<int64_t>(o.max_tokens, room);
  DeviceGuard dg(s->device);
  DecodeState h;
  std::memset(&h, 0, sizeof(h));
  h.pos = (int32_t)s->len;
  h.start_pos = (int32_t)s->len;
  h.active = 1;
  h.max_tokens = o.max_tokens;
  h.n_stop = o.n_stop;
  for (int i = 0; i < o.n_stop; ++i) h.stop_ids[i] = o.stop_ids[i];
  h.temperature = o.temperature;
  h.top_k = o.top_k;
  h.top_p = o.top_p;
  h.seed = o.seed;
  check(state_set_launch(s->st, h, s->stream), "state");
  capture_step_graph(s);
  const int64_t batch = 8;
  for (int64_t i = 0; i < steps; i += batch) {
    const int64_t nb = std::min(batch, steps - i);
    for (int64_t j = 0; j < nb; ++j) {
      CK(cudaGraphLaunch(s->step_graph, s->stream));
      count_launches(s->graph_kernels);
    }
    if (sync_host && o.n_stop > 0 && i + nb < steps) {
      int32_t done = 0;
      CK(cudaMemcpyAsync(&s->st_host->done, &s->st->done, sizeof(int32_t), cudaMemcpyDeviceToHost,
                         s->stream));
      CK(cudaStreamSynchronize(s->stream));
      done = s->st_host->done;
      if (done) break;
    }
  }
  (void)c;
  return steps;
}

int finish_generate(Session* s, const rpgc_gen_opts& o, int64_t steps, int32_t* out,
                    int32_t* n_out) {
  CK(cudaMemcpyAsync(s->st_host, s->st, sizeof(DecodeState), cudaMemcpyDeviceToHost, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  const DecodeState h = *s->st_host;
  if (h.error) {
    // the pending logits and the cache rows past len no longer match len:
    // the session needs a forward before its next generate
    s->has_logits = false;
    if (h.error & kErrBadToken) fail(RPGC_E_ARG, "a device-resident token id was outside the vocabulary");
    fail(RPGC_E_TIMEOUT, "a device wait gave up during generation (flags %d)", h.error);
  }
  if (h.n_gen < 0 || h.n_gen > steps) fail(RPGC_E_CUDA, "inconsistent decode state");
  if (h.n_gen > 0) CK(cudaMemcpy(out, s->gen_out, h.n_gen * sizeof(int32_t), cudaMemcpyDeviceToHost));
  *n_out = h.n_gen;
  s->len += h.n_gen;
  s->has_logits = true;
  if (!h.done && steps < o.max_tokens)
    fail(RPGC_E_CONTEXT_FULL, "context full after %d generated tokens (max_seq %lld)", h.n_gen,
         (long long)s->max_seq);
  return RPGC_OK;
}

template <typename F>
int guard(F&& f) {
  try {
    g_last_error.clear();
    return f();
  } catch (const Error& e) {
    g_last_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return RPGC_E_CUDA;
  } catch (...) {
    g_last_error = "unknown exception";
    return RPGC_E_CUDA;
  }
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

constexpr int32_t kMaxBatch = 256;

// Room for split-K partial sums of up to 8 partitions of the widest matrix
// per token: a few dozen session rows fill the GPU only with K split.
size_t batch_scratch_bytes(const rpgc_model_config& c, int32_t n) {
  const int64_t H = c.hidden, F = c.intermediate, qd = (int64_t)c.n_heads * c.head_dim;
  const int64_t kmax = std::max(H, std::max(qd, F));
  return gemm_scratch_bytes(n, kmax) + (size_t)n * 8 * (size_t)kmax * sizeof(float);
}

// The model's batch buffers, grown to hold n sessions (the caller holds
// bc.mu; the model's device is current; no batch is running).
void batch_buffers(Model* m, int32_t n) {
  BatchCache& bc = m->bcache;
  if (bc.cap >= n) return;
  bc.release();
  const int32_t cap = std::min<int32_t>(kMaxBatch, std::max<int32_t>(n, 8 * ((n + 7) / 8)));
  const rpgc_model_config& c = m->c;
  const size_t H = c.hidden, F = c.intermediate, V = c.vocab, qd = (size_t)c.n_heads * c.head_dim,
               kvd = (size_t)c.n_kv_heads * c.head_dim, N = (size_t)cap;
  auto alloc = [&](size_t bytes) {
    void* p = nullptr;
    CK(cudaMalloc(&p, bytes));
    bc.ptrs.push_back(p);
    return p;
  };
  bc.x = static_cast<float*>(alloc(N * H * 4));
  bc.h = static_cast<float*>(alloc(N * H * 4));
  bc.q = static_cast<float*>(alloc(N * qd * 4));
  bc.k = static_cast<float*>(alloc(N * kvd * 4));
  bc.v = static_cast<float*>(alloc(N * kvd * 4));
  bc.attn = static_cast<float*>(alloc(N * qd * 4));
  bc.gate = static_cast<float*>(alloc(N * F * 4));
  bc.up = static_cast<float*>(alloc(N * F * 4));
  bc.logits = static_cast<float*>(alloc(N * V * 4));
  bc.scratch = alloc(batch_scratch_bytes(c, cap));
  bc.states = static_cast<DecodeState**>(alloc(N * sizeof(DecodeState*)));
  bc.outs = static_cast<int32_t**>(alloc(N * sizeof(int32_t*)));
  bc.nouts = static_cast<int32_t**>(alloc(N * sizeof(int32_t*)));
  bc.dst = static_cast<float**>(alloc(N * sizeof(float*)));
  bc.entries = static_cast<AttnBatchEntry*>(alloc(N * sizeof(AttnBatchEntry)));
  bc.n_active = static_cast<int32_t*>(alloc(sizeof(int32_t)));
  CK(cudaMallocHost(&bc.n_active_host, sizeof(int32_t)));
  bc.cap = cap;
}

// Test hook (rpgc_test_stall_next_batch): index of the session whose
// attention waits time out in the next batched decode, -1 for none.
std::atomic<int32_t> g_test_stall{-1};

void batch_layers(const Model* m, int32_t n, float* x, float* q, float* k, float* v, float* attn, float* gate,
                  float* up, void* scratch, size_t sbytes, const AttnBatchEntry* entries, cudaStream_t cs) {
  const rpgc_model_config& c = m->c;
  const int64_t H = c.hidden, F = c.intermediate, qd = (int64_t)c.n_heads * c.head_dim,
                kvd = (int64_t)c.n_kv_heads * c.head_dim;
  for (int l = 0; l < c.n_layers; ++l) {
    const DevLayer& L = m->layers[l];
    const GemmGroupMat qkv[3] = {{L.q.type, L.q.w, L.q.rows, L.q.row_bytes, q, qd},
                                 {L.k.type, L.k.w, L.k.rows, L.k.row_bytes, k, kvd},
                                 {L.v.type, L.v.w, L.v.rows, L.v.row_bytes, v, kvd}};
    check(gemm_tc_split_norm(x, L.attn_norm, c.rms_eps, n, H, scratch, sbytes, cs), "norm split");
    check(gemm_tc_launch_group(qkv, 3, H, nullptr, n, scratch, sbytes, cs, true), "gemm qkv");
    AttnArgs aa{};
    aa.q = q;
    aa.k_new = k;
    aa.v_new = v;
    aa.out = attn;
    aa.n_heads = c.n_heads;
    aa.n_kv = c.n_kv_heads;
    aa.hd = c.head_dim;
    aa.q_norm = L.q_norm;
    aa.k_norm = L.k_norm;
    aa.rope = m->rope;
    aa.eps = c.rms_eps;
    aa.err = nullptr;  // each entry carries its session's error flags
    aa.batch = entries;
    aa.nbatch = n;
    aa.layer = l;
    check(attn_decode_launch(aa, cs), "attention");
    check(gemm_launch(L.o.type, L.o.w, L.o.rows, qd, L.o.row_bytes, attn, n, x, H, true, scratch, sbytes, cs),
          "gemm o");
    check(gemm_tc_split_norm(x, L.ffn_norm, c.rms_eps, n, H, scratch, sbytes, cs), "norm split");
    // gate and up share their input: one launch (at a few dozen rows each
    // alone would need split-K and a reduction to fill the GPU)
    const GemmGroupMat gu[2] = {{L.gate.type, L.gate.w, L.gate.rows, L.gate.row_bytes, gate, F},
                                {L.up.type, L.up.w, L.up.rows, L.up.row_bytes, up, F}};
    check(gemm_tc_launch_group(gu, 2, H, nullptr, n, scratch, sbytes, cs, true), "gemm gate+up");
    check(gemm_tc_split_glu(gate, up, n, F, scratch, sbytes, cs), "glu split");
    check(gemm_launch(L.down.type, L.down.w, L.down.rows, F, L.down.row_bytes, nullptr, n, x, H, true, scratch,
                      sbytes, cs, true),
          "gemm down");
  }
}

// The shapes batched decode needs: the tensor-core matmuls over the session
// rows (hidden, q width and FFN width multiples of 64, a supported type).
bool batch_shapes_ok(const Model* m) {
  const rpgc_model_config& c = m->c;
  const int64_t H = c.hidden, F = c.intermediate, qd = (int64_t)c.n_heads * c.head_dim;
  const int64_t kmax = std::max(H, std::max(qd, F));
  return m->tp_world == 1 && !m->layers.empty() && H % 64 == 0 && F % 64 == 0 && qd % 64 == 0 &&
         gemm_uses_tc(m->layers[0].q.type, 2, H, gemm_scratch_bytes(2, kmax));
}

// Batched multi-session decode: one step decodes one token for each session
// at once.  The sessions' rows share the weight stream: the matmuls run on
// the tensor cores over the session rows (the prefill kernels), the attention
// is the decode kernel with one grid slice per session (its own cache,
// position and state), the sampler one block per session.  Session i decodes
// with opts[i] (its own stop ids, sampling, seed and max_tokens: it goes
// inactive after its own count while the batch runs the largest).  The caller
// holds every session's lock and has checked pending logits and room for
// opts[i].max_tokens; afterwards every session's stream is ordered after the
// batch, and the caller finishes each session (finish_generate).
void batch_decode(const std::vector<Session*>& ss, const std::vector<rpgc_gen_opts>& opts) {
  const int32_t n = (int32_t)ss.size();
  Model* m = ss[0]->m;
  const rpgc_model_config& c = m->c;
  int32_t steps = 0;
  bool early = false;  // a session may go inactive before the last step
  for (const rpgc_gen_opts& o : opts) steps = std::max(steps, o.max_tokens);
  for (const rpgc_gen_opts& o : opts) early |= o.n_stop > 0 || o.max_tokens < steps;
  const int64_t H = c.hidden, V = c.vocab;
  if (!batch_shapes_ok(m))
    fail(RPGC_E_ARG, "batched decode needs the tensor-core matmul shapes (hidden, q width, FFN multiples of 64)");
  DeviceGuard dg(m->device);
  BatchCache& bc = m->bcache;
  std::lock_guard<std::mutex> blk(bc.mu);
  batch_buffers(m, n);
  const size_t sbytes = batch_scratch_bytes(c, n);
  cudaStream_t bs = ss[0]->stream;  // the batch runs on the first session's stream
  cudaEvent_t ev = nullptr;
  CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  struct EvGuard {
    cudaEvent_t e;
    ~EvGuard() { cudaEventDestroy(e); }
  } evg{ev};
  const int32_t stall = g_test_stall.exchange(-1);
  std::vector<DecodeState*> hs((size_t)n);
  std::vector<int32_t*> ho((size_t)n), hn((size_t)n);
  std::vector<float*> hd((size_t)n);
  std::vector<AttnBatchEntry> he((size_t)n);
  for (int32_t i = 0; i < n; ++i) {
    Session* s = ss[i];
    const rpgc_gen_opts& o = opts[(size_t)i];
    DecodeState st;
    std::memset(&st, 0, sizeof(st));
    st.pos = (int32_t)s->len;
    st.start_pos = (int32_t)s->len;
    st.active = 1;
    st.max_tokens = o.max_tokens;
    st.n_stop = o.n_stop;
    for (int j = 0; j < o.n_stop; ++j) st.stop_ids[j] = o.stop_ids[j];
    st.temperature = o.temperature;
    st.top_k = o.top_k;
    st.top_p = o.top_p;
    st.seed = o.seed;
    check(state_set_launch(s->st, st, s->stream), "state");
    CK(cudaEventRecord(ev, s->stream));  // the session's own work comes first
    CK(cudaStreamWaitEvent(bs, ev, 0));
    CK(cudaMemcpyAsync(bc.logits + (size_t)i * V, s->logits, V * sizeof(float), cudaMemcpyDeviceToDevice, bs));
    hs[i] = s->st;
    ho[i] = s->gen_out;
    hn[i] = s->n_out;
    hd[i] = s->logits;
    he[i] = AttnBatchEntry{s->st, s->kc, s->vc, s->max_seq, &s->st->error, i == stall ? 1 : 0};
  }
  // the session table of this batch, ordered on the batch stream (the
  // previous batch on these buffers has finished: its callers synchronised)
  CK(cudaMemcpyAsync(bc.states, hs.data(), n * sizeof(DecodeState*), cudaMemcpyHostToDevice, bs));
  CK(cudaMemcpyAsync(bc.outs, ho.data(), n * sizeof(int32_t*), cudaMemcpyHostToDevice, bs));
  CK(cudaMemcpyAsync(bc.nouts, hn.data(), n * sizeof(int32_t*), cudaMemcpyHostToDevice, bs));
  CK(cudaMemcpyAsync(bc.dst, hd.data(), n * sizeof(float*), cudaMemcpyHostToDevice, bs));
  CK(cudaMemcpyAsync(bc.entries, he.data(), n * sizeof(AttnBatchEntry), cudaMemcpyHostToDevice, bs));
  CK(cudaStreamSynchronize(bs));  // the pageable host tables are read before they go
  SampleArgs sa{};
  sa.logits = bc.logits;
  sa.n = V;
  sa.embd = m->embd.w;
  sa.embd_row_bytes = m->embd.row_bytes;
  sa.embd_type = m->embd.type;
  sa.hidden = (int32_t)H;
  sa.x = bc.x;
  sa.states = bc.states;
  sa.out_ids_b = bc.outs;
  sa.n_out_b = bc.nouts;
  sa.nbatch = n;
  auto one_step = [&] {
    check(sample_launch(sa, bs), "sample");
    batch_layers(m, n, bc.x, bc.q, bc.k, bc.v, bc.attn, bc.gate, bc.up, bc.scratch, sbytes, bc.entries, bs);
    check(rmsnorm_rows_launch(bc.x, m->out_norm, n, c.hidden, c.rms_eps, bc.h, bs), "rmsnorm");
    check(gemm_launch(m->lm_head.type, m->lm_head.w, m->lm_head.rows, H, m->lm_head.row_bytes, bc.h, n, bc.logits,
                      V, false, bc.scratch, sbytes, bs),
          "gemm lm_head");
    check(commit_rows_launch(bc.logits, V, bc.dst, bc.states, n, bs), "commit logits");
  };
  // Every argument of a step (positions, states, buffers) lives on the
  // device, so one captured graph of a step serves every step of every batch
  // of this size on these buffers (~13 launches per layer cost one).  The
  // first batch of a size runs its first step as plain launches (one-time
  // kernel attributes are set there) and captures the graph after it.
  int32_t done_steps = 0;
  auto it = bc.graphs.find(n);
  if (it == bc.graphs.end()) {
    one_step();
    done_steps = 1;
    if (steps > 1) {
      cudaGraph_t g = nullptr;
      int64_t nk = 0;
      CK(cudaStreamBeginCapture(bs, cudaStreamCaptureModeThreadLocal));
      t_capture_count = &nk;
      try {
        one_step();
      } catch (...) {
        t_capture_count = nullptr;
        cudaStreamEndCapture(bs, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      t_capture_count = nullptr;
      CK(cudaStreamEndCapture(bs, &g));
      BatchCache::StepGraph sg;
      const cudaError_t e = cudaGraphInstantiate(&sg.exec, g, 0);
      cudaGraphDestroy(g);
      CK(e);
      sg.kernels = nk;
      it = bc.graphs.emplace(n, sg).first;
    }
  }
  // Replays; with stop ids or unequal lengths, every 8 steps the host reads
  // how many sessions are still active and ends the batch once none is.
  for (int32_t step = done_steps; step < steps;) {
    const int32_t nb = std::min<int32_t>(8, steps - step);
    for (int32_t j = 0; j < nb; ++j) {
      CK(cudaGraphLaunch(it->second.exec, bs));
      count_launches(it->second.kernels);
    }
    step += nb;
    if (early && step < steps) {
      check(count_active_launch(bc.states, n, bc.n_active, bs), "count active");
      CK(cudaMemcpyAsync(bc.n_active_host, bc.n_active, sizeof(int32_t), cudaMemcpyDeviceToHost, bs));
      CK(cudaStreamSynchronize(bs));
      if (*bc.n_active_host == 0) break;
    }
  }
  CK(cudaEventRecord(ev, bs));
  for (int32_t i = 0; i < n; ++i) CK(cudaStreamWaitEvent(ss[i]->stream, ev, 0));
  CK(cudaStreamSynchronize(bs));  // the buffers serve the next batch only after this one
}

// One rpgc_generate call waiting to join a batch (rpgc_model_set_batching).
struct BatchRequest {
  Session* s = nullptr;
  rpgc_gen_opts o{};
  int32_t* out = nullptr;
  int32_t* n_out = nullptr;
  bool done = false;  // set by the caller that ran its batch, under the batcher's lock
  int code = RPGC_OK;
  std::string msg;
};

// Runs a gathered batch; each request records its own outcome.  One request
// alone decodes as an unbatched rpgc_generate (the persistent step kernel).
void serve_batch(const std::vector<BatchRequest*>& batch) {
  auto record_all = [&](int code, const char* msg) {
    for (BatchRequest* r : batch) {
      r->code = code;
      r->msg = msg;
    }
  };
  auto run = [](BatchRequest* r, auto&& f) {
    try {
      f();
    } catch (const Error& e) {
      r->code = e.code;
      r->msg = e.what();
    } catch (const std::exception& e) {
      r->code = RPGC_E_CUDA;
      r->msg = e.what();
    } catch (...) {
      r->code = RPGC_E_CUDA;
      r->msg = "unknown exception";
    }
  };
  if (batch.size() == 1) {
    BatchRequest* r = batch[0];
    run(r, [&] {
      std::lock_guard<std::mutex> lk(r->s->mu);
      const int64_t steps = generate(r->s, r->o, true);
      finish_generate(r->s, r->o, steps, r->out, r->n_out);
    });
    return;
  }
  std::vector<Session*> ss;
  std::vector<rpgc_gen_opts> opts;
  for (BatchRequest* r : batch) {
    ss.push_back(r->s);
    opts.push_back(r->o);
  }
  std::vector<Session*> order(ss);  // lock in address order (no lock-order inversion)
  std::sort(order.begin(), order.end());
  std::vector<std::unique_lock<std::mutex>> locks;
  for (Session* s : order) locks.emplace_back(s->mu);
  try {
    DeviceGuard dg(ss[0]->m->device);
    for (size_t i = 0; i < ss.size(); ++i)
      if (!ss[i]->has_logits || ss[i]->max_seq - ss[i]->len < opts[i].max_tokens)
        fail(RPGC_E_STATE, "a session of the batch changed while it waited");
    batch_decode(ss, opts);
    for (size_t i = 0; i < ss.size(); ++i)
      run(batch[i], [&] { finish_generate(ss[i], opts[i], opts[i].max_tokens, batch[i]->out, batch[i]->n_out); });
    cudaStreamSynchronize(ss[0]->stream);
  } catch (const Error& e) {
    record_all(e.code, e.what());
  } catch (const std::exception& e) {
    record_all(RPGC_E_CUDA, e.what());
  } catch (...) {
    record_all(RPGC_E_CUDA, "unknown exception");
  }
}

// Whether an rpgc_generate call joins its model's batches: batching on, the
// model batchable, valid options, pending logits and room for max_tokens (a
// call that fails any of these runs unbatched, which reports its errors).
bool batch_eligible(Session* s, const rpgc_gen_opts& o) {
  Model* m = s->m;
  {
    std::lock_guard<std::mutex> lk(m->batcher.mu);
    if (m->batcher.max_batch < 2) return false;
  }
  if (!batch_shapes_ok(m)) return false;
  if (o.max_tokens <= 0 || o.n_stop < 0 || o.n_stop > RPGC_MAX_STOP || (o.n_stop > 0 && !o.stop_ids)) return false;
  std::lock_guard<std::mutex> lk(s->mu);
  return s->has_logits && s->max_seq - s->len >= o.max_tokens;
}

// rpgc_generate with batching on: the call queues its request; the first
// caller to find no batch running leads: it waits up to the window (or until
// max_batch requests of distinct sessions are queued), takes them in arrival
// order with its own first, runs them as one batch and wakes the others.
// Requests left over lead the next batch.
int batched_generate(Session* s, const rpgc_gen_opts& o, int32_t* out, int32_t* n_out) {
  Batcher& b = s->m->batcher;
  BatchRequest r;
  r.s = s;
  r.o = o;
  r.out = out;
  r.n_out = n_out;
  std::unique_lock<std::mutex> lk(b.mu);
  b.pending.push_back(&r);
  b.cv.notify_all();
  while (!r.done && b.leading) b.cv.wait(lk);
  if (!r.done) {
    b.leading = true;
    const int32_t maxb = std::max<int32_t>(2, b.max_batch);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(b.window_us);
    b.cv.wait_until(lk, deadline, [&] { return (int32_t)b.pending.size() >= maxb; });
    std::vector<BatchRequest*> batch{&r};
    b.pending.erase(std::find(b.pending.begin(), b.pending.end(), &r));
    for (auto it = b.pending.begin(); it != b.pending.end() && (int32_t)batch.size() < maxb;) {
      bool dup = false;  // one call at a time per session: a second one waits for the next batch
      for (BatchRequest* q : batch) dup |= q->s == (*it)->s;
      if (dup) {
        ++it;
        continue;
      }
      batch.push_back(*it);
      it = b.pending.erase(it);
    }
    if (batch.size() > 1) {
      b.batches += 1;
      b.requests += (int64_t)batch.size();
    }
    lk.unlock();
    try {  // every request gets an outcome, and leadership is always handed back
      serve_batch(batch);
    } catch (...) {
      for (BatchRequest* q : batch) {
        q->code = RPGC_E_CUDA;
        q->msg = "batched decode failed before it started";
      }
    }
    lk.lock();
    for (BatchRequest* q : batch) q->done = true;
    b.leading = false;
    b.cv.notify_all();
  }
  if (r.code != RPGC_OK) throw Error(r.code, r.msg);
  return RPGC_OK;
}

}  // namespace

// Lets other translation units of the library report through rpgc_last_error().
void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

void count_launches(int64_t k) {
  if (t_capture_count) *t_capture_count += k;
  else g_launches.fetch_add(k, std::memory_order_relaxed);
}
int64_t launches_enqueued() { return g_launches.load(std::memory_order_relaxed); }

}  // namespace rpgc

using namespace rpgc;

extern "C" {

const char* rpgc_version(void) { return "0.1.0-b200"; }

int64_t rpgc_kernel_launches(void) { return launches_enqueued(); }
const char* rpgc_last_error(void) { return g_last_error.c_str(); }

int rpgc_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int32_t rpgc_model_upload(int device, const rpgc_model_config* cfg, const rpgc_tensor* tensors,
                          int32_t n_tensors) {
  return guard([&] {
    if (!cfg || !tensors || n_tensors <= 0) fail(RPGC_E_ARG, "null config or tensor table");
    return upload(device, *cfg, tensors, n_tensors);
  });
}

int rpgc_tp_id(void* id, int64_t bytes) {
  return guard([&] {
    if (!id || bytes < (int64_t)sizeof(ncclUniqueId)) fail(RPGC_E_ARG, "id buffer under %d bytes", (int)sizeof(ncclUniqueId));
    const NcclApi* api = nccl_api();
    if (!api) fail(RPGC_E_STATE, "tensor parallelism needs libnccl.so.2");
    ncclUniqueId u;
    const ncclResult_t r = api->get_id(&u);
    if (r != ncclSuccess) fail(RPGC_E_CUDA, "ncclGetUniqueId: %s", api->error_string(r));
    std::memcpy(id, &u, sizeof(u));
    return RPGC_OK;
  });
}

int rpgc_tp_shard_of(const rpgc_model_config* cfg, int32_t rank, int32_t world, rpgc_tp_shard* out) {
  return guard([&] {
    if (!cfg || !out) fail(RPGC_E_ARG, "null argument");
    *out = tp_shard_of(*cfg, rank, world);
    return RPGC_OK;
  });
}

int32_t rpgc_model_upload_tp(int device, const rpgc_model_config* cfg, const rpgc_tensor* tensors,
                             int32_t n_tensors, int32_t rank, int32_t world, const void* id) {
  return guard([&] {
    if (!cfg || !tensors || n_tensors <= 0) fail(RPGC_E_ARG, "null config or tensor table");
    return upload(device, *cfg, tensors, n_tensors, rank, world, id);
  });
}

int32_t rpgc_model_load_gguf(int device, const char* path, int32_t max_pos) {
  return guard([&] {
    if (!path || !*path) fail(RPGC_E_ARG, "empty path");
    GgufReader r;
    try {
      r.Open(path);
    } catch (const std::exception& e) {
      fail(RPGC_E_IO, "%s", e.what());
    }
    const std::string arch = r.Str("general.architecture", "");
    if (arch != "qwen3") fail(RPGC_E_ARG, "architecture is '%s'; only qwen3 is implemented", arch.c_str());
    rpgc_model_config c{};
    const std::string a = arch + ".";
    c.n_layers = (int32_t)r.Int(a + "block_count", 0);
    c.hidden = (int32_t)r.Int(a + "embedding_length", 0);
    c.n_heads = (int32_t)r.Int(a + "attention.head_count", 0);
    c.n_kv_heads = (int32_t)r.Int(a + "attention.head_count_kv", c.n_heads);
    c.intermediate = (int32_t)r.Int(a + "feed_forward_length", 0);
    c.context_length = (int32_t)r.Int(a + "context_length", 4096);
    if (c.context_length <= 0) c.context_length = 4096;
    const int64_t key_len = r.Int(a + "attention.key_length", 0);
    c.head_dim = key_len > 0 ? (int32_t)key_len : (c.n_heads > 0 ? c.hidden / c.n_heads : 0);
    if (r.Int(a + "attention.value_length", c.head_dim) != c.head_dim)
      fail(RPGC_E_ARG, "value_length differs from key_length");
    c.rope_theta = (float)r.Float(a + "rope.freq_base", 10000.0);
    c.rms_eps = (float)r.Float(a + "attention.layer_norm_rms_epsilon", 1e-6);
    const size_t vocab = r.ArrayLen("tokenizer.ggml.tokens");
    c.vocab = (int32_t)vocab;
    c.max_pos = max_pos > 0 ? max_pos : 4096;
    std::vector<rpgc_tensor> tab;
    std::vector<std::string> names;
    names.reserve(r.tensors().size());
    for (const auto& t : r.tensors()) names.push_back(t.name);
    size_t i = 0;
    for (const auto& t : r.tensors()) {
      rpgc_tensor x{};
      x.name = names[i++].c_str();
      x.type = t.type;
      x.n_dims = (int32_t)t.dims.size();
      for (size_t d = 0; d < t.dims.size(); ++d) x.dims[d] = t.dims[d];
      x.data = r.TensorData(t);
      x.n_bytes = t.n_bytes;
      tab.push_back(x);
    }
    if (vocab == 0) {  // fall back to the embedding's rows when no token list
      for (const auto& x : tab)
        if (std::string(x.name) == "token_embd.weight" && x.n_dims == 2) c.vocab = (int32_t)x.dims[1];
    }
    const int32_t eos = (int32_t)r.Int("tokenizer.ggml.eos_token_id", -1);
    int32_t im_end = -1;  // Tokenizer::IdOf("<|im_end|>") over the vocabulary
    if (const GgufValue* tv = r.Find("tokenizer.ggml.tokens"))
      for (size_t k = 0; k < tv->strs.size(); ++k)
        if (tv->strs[k] == "<|im_end|>") {
          im_end = (int32_t)k;
          break;
        }
    const int32_t h = upload(device, c, tab.data(), (int32_t)tab.size());
    std::lock_guard<std::mutex> lk(g_mu);
    Model* m = model_locked(h);
    m->eos_id = eos >= 0 && eos < c.vocab ? eos : -1;
    m->im_end_id = im_end < c.vocab ? im_end : -1;
    return h;
  });
}

int rpgc_model_set_special_ids(int32_t model, int32_t eos_id, int32_t im_end_id) {
  return guard([&] {
    std::lock_guard<std::mutex> lk(g_mu);
    Model* m = model_locked(model);
    if (eos_id < -1 || eos_id >= m->c.vocab || im_end_id < -1 || im_end_id >= m->c.vocab)
      fail(RPGC_E_ARG, "special ids %d, %d outside -1 .. %d", eos_id, im_end_id, m->c.vocab - 1);
    m->eos_id = eos_id;
    m->im_end_id = im_end_id;
    return RPGC_OK;
  });
}

int rpgc_model_special_ids(int32_t model, int32_t* eos_id, int32_t* im_end_id) {
  return guard([&] {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!eos_id || !im_end_id) fail(RPGC_E_ARG, "null output");
    const Model* m = model_locked(model);
    *eos_id = m->eos_id;
    *im_end_id = m->im_end_id;
    return RPGC_OK;
  });
}

int rpgc_model_get_config(int32_t model, rpgc_model_config* out) {
  return guard([&] {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!out) fail(RPGC_E_ARG, "null output");
    Model* m = model_locked(model);
    *out = m->cg;
    out->max_pos = (int32_t)m->n_rope;
    return RPGC_OK;
  });
}

int64_t rpgc_model_weight_bytes(int32_t model) {
  int64_t v = 0;
  const int rc = guard([&] {
    std::lock_guard<std::mutex> lk(g_mu);
    v = model_locked(model)->weight_bytes;
    return RPGC_OK;
  });
  return rc == RPGC_OK ? v : rc;
}

int rpgc_model_free(int32_t model) {
  return guard([&] {
    std::unique_ptr<Model> m;
    std::vector<std::unique_ptr<Session>> dead;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_models.find(model);
      if (it == g_models.end()) return RPGC_OK;  // invalid handle: no-op
      for (int32_t s : it->second->sessions) {
        auto si = g_sessions.find(s);
        if (si != g_sessions.end()) {
          dead.push_back(std::move(si->second));
          g_sessions.erase(si);
        }
      }
      m = std::move(it->second);
      g_models.erase(it);
    }
    dead.clear();
    m.reset();
    return RPGC_OK;
  });
}

int32_t rpgc_session_create(int32_t model, int32_t max_seq) {
  return guard([&] { return session_create(model, max_seq); });
}

int rpgc_session_destroy(int32_t session) {
  return guard([&] {
    std::unique_ptr<Session> s;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_sessions.find(session);
      if (it == g_sessions.end()) return RPGC_OK;
      auto mi = g_models.find(it->second->model_id);
      if (mi != g_models.end()) {
        auto& v = mi->second->sessions;
        for (size_t i = 0; i < v.size(); ++i)
          if (v[i] == session) {
            v.erase(v.begin() + i);
            break;
          }
      }
      s = std::move(it->second);
      g_sessions.erase(it);
    }
    std::lock_guard<std::mutex> lk2(s->mu);
    return RPGC_OK;
  });
}

int64_t rpgc_session_len(int32_t session) {
  int64_t v = 0;
  const int rc = guard([&] {
    v = require_session(session)->len;
    return RPGC_OK;
  });
  return rc == RPGC_OK ? v : rc;
}

int rpgc_session_set_len(int32_t session, int64_t len) {
  return guard([&] {
    Session* s = require_session(session);
    std::lock_guard<std::mutex> lk(s->mu);
    if (len < 0 || len > s->max_seq)
      fail(RPGC_E_ARG, "length %lld out of range (capacity %lld)", (long long)len, (long long)s->max_seq);
    s->len = len;
    s->has_logits = false;
    return RPGC_OK;
  });
}

int rpgc_session_copy_prefix(int32_t dst, int32_t src, int64_t n) {
  return guard([&] {
    Session* d = require_session(dst);
    Session* s = require_session(src);
    if (d == s) fail(RPGC_E_ARG, "source and destination are the same session");
    if (d->m != s->m) fail(RPGC_E_ARG, "the sessions belong to different models");
    std::scoped_lock lk(d->mu, s->mu);
    if (n < 0 || n > s->len)
      fail(RPGC_E_ARG, "prefix of %lld positions, the source holds %lld", (long long)n, (long long)s->len);
    if (n > d->max_seq)
      fail(RPGC_E_CONTEXT_FULL, "prefix of %lld positions, capacity %lld", (long long)n, (long long)d->max_seq);
    DeviceGuard dg(d->device);
    if (n > 0) {
      // rows [0, n) of every (layer, kv head) block: one strided copy per cache,
      // ordered after the source's writes and before its next ones
      const Model* m = d->m;
      const size_t hd = (size_t)m->c.head_dim, blocks = (size_t)m->c.n_layers * m->c.n_kv_heads;
      const size_t wbytes = (size_t)n * hd * sizeof(float);
      cudaEvent_t ev = nullptr;
      CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
      CK(cudaEventRecord(ev, s->stream));
      CK(cudaStreamWaitEvent(d->stream, ev, 0));
      CK(cudaMemcpy2DAsync(d->kc, (size_t)d->max_seq * hd * sizeof(float), s->kc,
                           (size_t)s->max_seq * hd * sizeof(float), wbytes, blocks,
                           cudaMemcpyDeviceToDevice, d->stream));
      CK(cudaMemcpy2DAsync(d->vc, (size_t)d->max_seq * hd * sizeof(float), s->vc,
                           (size_t)s->max_seq * hd * sizeof(float), wbytes, blocks,
                           cudaMemcpyDeviceToDevice, d->stream));
      CK(cudaEventRecord(ev, d->stream));
      CK(cudaStreamWaitEvent(s->stream, ev, 0));
      CK(cudaEventDestroy(ev));
    }
    d->len = n;
    d->has_logits = false;
    return RPGC_OK;
  });
}

void* rpgc_session_stream(int32_t session) {
  void* p = nullptr;
  guard([&] {
    p = require_session(session)->stream;
    return RPGC_OK;
  });
  return p;
}

int rpgc_session_read_kv(int32_t session, float* k, float* v) {
  return guard([&] {
    Session* s = require_session(session);
    std::lock_guard<std::mutex> lk(s->mu);
    DeviceGuard dg(s->device);
    const size_t bytes = (size_t)s->m->c.n_layers * s->layer_cache_floats() * sizeof(float);
    if (k) CK(cudaMemcpyAsync(k, s->kc, bytes, cudaMemcpyDeviceToHost, s->stream));
    if (v) CK(cudaMemcpyAsync(v, s->vc, bytes, cudaMemcpyDeviceToHost, s->stream));
    CK(cudaStreamSynchronize(s->stream));
    return RPGC_OK;
  });
}

int rpgc_forward(int32_t session, const int32_t* ids, int64_t n, float* last_logits,
                 float* all_logits) {
  return guard([&] {
    if (!ids) fail(RPGC_E_ARG, "null ids");
    Session* s = require_session(session);
    std::lock_guard<std::mutex> lk(s->mu);
    forward(s, ids, false, n, last_logits, all_logits);
    return RPGC_OK;
  });
}

int rpgc_forward_device(int32_t session, const int32_t* ids_dev, int64_t n) {
  return guard([&] {
    if (!ids_dev) fail(RPGC_E_ARG, "null ids");
    Session* s = require_session(session);
    std::lock_guard<std::mutex> lk(s->mu);
    forward(s, ids_dev, true, n, nullptr, nullptr);
    return RPGC_OK;
  });
}

int rpgc_generate(int32_t session, const rpgc_gen_opts* opts, int32_t* out_ids, int32_t* n_out) {
  return guard([&] {
    if (!opts || !out_ids || !n_out) fail(RPGC_E_ARG, "null argument");
    *n_out = 0;
    Session* s = require_session(session);
    if (batch_eligible(s, *opts)) return batched_generate(s, *opts, out_ids, n_out);
    std::lock_guard<std::mutex> lk(s->mu);
    const int64_t steps = generate(s, *opts, true);
    return finish_generate(s, *opts, steps, out_ids, n_out);
  });
}

// Batched multi-session decode with one set of options (batch_decode).
int rpgc_generate_batch(const int32_t* sessions, int32_t n, const rpgc_gen_opts* opts, int32_t* out_ids,
                        int32_t* n_out) {
  return guard([&] {
    if (!sessions || !opts || !out_ids || !n_out) fail(RPGC_E_ARG, "null argument");
    if (n < 1 || n > kMaxBatch) fail(RPGC_E_ARG, "batch of %d sessions (1 .. %d)", n, kMaxBatch);
    const rpgc_gen_opts& o = *opts;
    if (o.max_tokens <= 0) fail(RPGC_E_ARG, "max_tokens must be positive, got %d", o.max_tokens);
    if (o.n_stop < 0 || o.n_stop > RPGC_MAX_STOP) fail(RPGC_E_ARG, "at most %d stop ids", RPGC_MAX_STOP);
    if (o.n_stop > 0 && !o.stop_ids) fail(RPGC_E_ARG, "stop_ids is NULL");
    for (int32_t i = 0; i < n; ++i) n_out[i] = 0;
    std::vector<Session*> ss((size_t)n);
    for (int32_t i = 0; i < n; ++i) {
      ss[i] = require_session(sessions[i]);
      for (int32_t j = 0; j < i; ++j)
        if (ss[j] == ss[i]) fail(RPGC_E_ARG, "session %d appears twice in the batch", sessions[i]);
      if (ss[i]->m != ss[0]->m) fail(RPGC_E_ARG, "the sessions of a batch must share one model");
    }
    const Model* m = ss[0]->m;
    if (m->tp_world > 1) fail(RPGC_E_ARG, "tensor-parallel models decode one session at a time");
    std::vector<Session*> order(ss);  // lock in address order (no lock-order inversion)
    std::sort(order.begin(), order.end());
    std::vector<std::unique_lock<std::mutex>> locks;
    for (Session* s : order) locks.emplace_back(s->mu);
    for (int32_t i = 0; i < n; ++i) {
      if (!ss[i]->has_logits) fail(RPGC_E_STATE, "session %d has no pending logits: call rpgc_forward first", sessions[i]);
      if (ss[i]->max_seq - ss[i]->len < o.max_tokens)
        fail(RPGC_E_CONTEXT_FULL, "session %d has room for %lld more tokens, max_tokens is %d", sessions[i],
             (long long)(ss[i]->max_seq - ss[i]->len), o.max_tokens);
    }
    DeviceGuard dg(m->device);
    batch_decode(ss, std::vector<rpgc_gen_opts>((size_t)n, o));
    // every session is finished with its own outcome; the call reports the
    // first failure (n_out of a failed session stays 0, its length unchanged)
    int code = RPGC_OK;
    std::string msg;
    for (int32_t i = 0; i < n; ++i) {
      try {
        finish_generate(ss[i], o, o.max_tokens, out_ids + (size_t)i * o.max_tokens, n_out + i);
      } catch (const Error& e) {
        n_out[i] = 0;
        if (code == RPGC_OK) {
          code = e.code;
          msg = "session " + std::to_string(sessions[i]) + ": " + e.what();
        }
      }
    }
    CK(cudaStreamSynchronize(ss[0]->stream));
    if (code != RPGC_OK) throw Error(code, msg);
    return RPGC_OK;
  });
}

int rpgc_model_set_batching(int32_t model, int32_t max_batch, int32_t window_us) {
  return guard([&] {
    if (max_batch < 0 || max_batch > kMaxBatch) fail(RPGC_E_ARG, "max_batch %d outside 0 .. %d", max_batch, kMaxBatch);
    if (window_us < 0 || window_us > 1000000) fail(RPGC_E_ARG, "window_us %d outside 0 .. 1000000", window_us);
    Model* m = nullptr;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      m = model_locked(model);
    }
    if (max_batch > 1 && !batch_shapes_ok(m))
      fail(RPGC_E_ARG, "this model cannot batch sessions (tensor-parallel, or not the tensor-core matmul shapes)");
    std::lock_guard<std::mutex> lk(m->batcher.mu);
    m->batcher.max_batch = max_batch > 1 ? max_batch : 0;
    m->batcher.window_us = window_us;
    return RPGC_OK;
  });
}

int rpgc_model_batching_stats(int32_t model, int64_t* batches, int64_t* requests) {
  return guard([&] {
    if (!batches || !requests) fail(RPGC_E_ARG, "null argument");
    Model* m = nullptr;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      m = model_locked(model);
    }
    std::lock_guard<std::mutex> lk(m->batcher.mu);
    *batches = m->batcher.batches;
    *requests = m->batcher.requests;
    return RPGC_OK;
  });
}

int rpgc_test_stall_next_batch(int32_t index) {
  return guard([&] {
    if (index < -1 || index >= kMaxBatch) fail(RPGC_E_ARG, "index %d outside -1 .. %d", index, kMaxBatch - 1);
    g_test_stall.store(index);
    return RPGC_OK;
  });
}

int rpgc_generate_device(int32_t session, const rpgc_gen_opts* opts, int32_t* out_ids_dev,
                         int32_t* n_out_dev) {
  return guard([&] {
    if (!opts || !out_ids_dev || !n_out_dev) fail(RPGC_E_ARG, "null argument");
    if (opts->n_stop != 0)
      fail(RPGC_E_ARG, "device-resident generation runs a fixed number of steps: no stop ids");
    Session* s = require_session(session);
    std::lock_guard<std::mutex> lk(s->mu);
    const int64_t steps = generate(s, *opts, false);
    if (steps < opts->max_tokens)
      fail(RPGC_E_CONTEXT_FULL, "max_tokens %d exceeds the remaining context", opts->max_tokens);
    DeviceGuard dg(s->device);
    CK(cudaMemcpyAsync(out_ids_dev, s->gen_out, steps * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                       s->stream));
    CK(cudaMemcpyAsync(n_out_dev, s->n_out, sizeof(int32_t), cudaMemcpyDeviceToDevice, s->stream));
    s->len += steps;
    s->has_logits = true;
    return RPGC_OK;
  });
}

int rpgc_session_sync(int32_t session) {
  return guard([&] {
    Session* s = require_session(session);
    DeviceGuard dg(s->device);
    CK(cudaStreamSynchronize(s->stream));
    CK(cudaMemcpy(s->st_host, s->st, sizeof(DecodeState), cudaMemcpyDeviceToHost));
    if (s->st_host->error & kErrBadToken) {  // reported once
      const int32_t zero = 0;
      CK(cudaMemcpy(&s->st->error, &zero, sizeof(zero), cudaMemcpyHostToDevice));
      fail(RPGC_E_ARG, "a device-resident token id was outside the vocabulary (embedded as zeros)");
    }
    if (s->st_host->error) fail(RPGC_E_TIMEOUT, "a device wait gave up (flags %d)", s->st_host->error);
    return RPGC_OK;
  });
}

int rpgc_dequantize_rows(uint32_t type, const void* w, int64_t rows, int64_t cols, float* out,
                         void* stream) {
  return guard([&] {
    const int64_t rb = row_bytes_of(type, cols);
    if (!w || !out || rows <= 0 || rb < 0 || (type != RPGC_F16 && !kernel_type(type)))
      fail(RPGC_E_ARG, "bad dequantize arguments (type %u, %lld x %lld)", type, (long long)rows,
           (long long)cols);
    check(dequant_launch(type, static_cast<const uint8_t*>(w), rows, cols, rb, out, as_stream(stream)),
          "dequant");
    return RPGC_OK;
  });
}

int rpgc_matvec(uint32_t type, const void* w, int64_t rows, int64_t cols, const float* x, float* y,
                void* stream) {
  return guard([&] {
    const int64_t rb = row_bytes_of(type, cols);
    if (!w || !x || !y || rows <= 0 || rb < 0 || !kernel_type(type) || cols % 32)
      fail(RPGC_E_ARG, "bad matvec arguments (type %u, %lld x %lld)", type, (long long)rows,
           (long long)cols);
    if (reinterpret_cast<uintptr_t>(w) & 15) fail(RPGC_E_ARG, "weights must be 16-byte aligned");
    if (!gemv_supported(cols, false)) {  // input length outside the decode kernel: CUDA-core GEMM
      check(gemm_launch(type, static_cast<const uint8_t*>(w), rows, cols, rb, x, 1, y, rows, false,
                        nullptr, 0, as_stream(stream)),
            "matvec");
      return RPGC_OK;
    }
    GemvArgs g{};
    g.seg[0].w = static_cast<const uint8_t*>(w);
    g.seg[0].out = y;
    g.seg[0].rows = rows;
    g.seg[0].row_bytes = rb;
    g.seg[0].type = type;
    g.seg[0].mode = kStore;
    g.nseg = 1;
    g.K = (int32_t)cols;
    g.x = x;
    check(gemv_launch(g, as_stream(stream), false), "gemv");
    return RPGC_OK;
  });
}

int rpgc_matmul(uint32_t type, const void* w, int64_t rows, int64_t cols, const float* X, int64_t n,
                float* OUT, void* stream) {
  if (n == 1) return rpgc_matvec(type, w, rows, cols, X, OUT, stream);
  return guard([&] {
    const int64_t rb = row_bytes_of(type, cols);
    if (!w || !X || !OUT || rows <= 0 || n <= 0 || rb < 0 || !kernel_type(type) || cols % 32)
      fail(RPGC_E_ARG, "bad matmul arguments");
    cudaStream_t cs = as_stream(stream);
    const size_t sb = gemm_scratch_bytes(n, cols);
    void* scratch = nullptr;
    CK(cudaMallocAsync(&scratch, sb, cs));
    const cudaError_t e = gemm_launch(type, static_cast<const uint8_t*>(w), rows, cols, rb, X, n, OUT,
                                      rows, false, scratch, sb, cs);
    cudaFreeAsync(scratch, cs);
    check(e, "gemm");
    return RPGC_OK;
  });
}

int rpgc_attention_decode(const float* q, const float* k_cache, const float* v_cache,
                          int64_t max_seq, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                          int64_t pos, float* out, void* stream) {
  return guard([&] {
    if (!q || !k_cache || !v_cache || !out || n_heads <= 0 || n_kv_heads <= 0 || max_seq <= 0)
      fail(RPGC_E_ARG, "bad attention arguments");
    const int32_t grp = n_heads % n_kv_heads ? 0 : n_heads / n_kv_heads;
    if (head_dim != 128 || !(grp == 1 || grp == 2 || grp == 4 || grp == 8))
      fail(RPGC_E_ARG, "attention takes head_dim 128 and a GQA group of 1, 2, 4 or 8");
    if (pos < 0 || pos >= max_seq || pos > INT32_MAX - 1) fail(RPGC_E_ARG, "pos out of range");
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
      fail(RPGC_E_ARG, "caches must be 16-byte aligned");
    cudaStream_t cs = as_stream(stream);
    AttnArgs a{};
    a.q = q;
    a.kc = k_cache;
    a.vc = v_cache;
    a.out = out;
    a.max_seq = max_seq;
    a.n_heads = n_heads;
    a.n_kv = n_kv_heads;
    a.hd = head_dim;
    a.pos0 = pos;
    a.n = 1;
    check(attn_decode_launch(a, cs), "attention decode");
    return RPGC_OK;
  });
}

int rpgc_sample(const float* logits, int64_t n, float temperature, int32_t top_k, float top_p,
                float u, int32_t* token_dev, void* stream) {
  return guard([&] {
    if (!logits || !token_dev || n <= 0) fail(RPGC_E_ARG, "bad sample arguments");
    SampleArgs a{};
    a.logits = logits;
    a.n = n;
    a.temperature = temperature;
    a.top_k = top_k;
    a.top_p = top_p;
    a.u = u;
    a.token_out = token_dev;
    check(sample_launch(a, as_stream(stream)), "sample");
    return RPGC_OK;
  });
}

}  // extern "C"
