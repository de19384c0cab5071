// ref_driver.cc -- extern "C" shim over the reference's own C++ token loop.
//
// TEST INFRASTRUCTURE ONLY.  It is compiled together with the reference's
// sources (read where they lie, never copied) into oracle/_ref/librpgref.so by
// oracle/Makefile, and exists so that Python tests and the bench's CPU
// baseline can call the reference's internal entry points, which its public C
// ABI (include/rpg_engine.h) does not expose:
//   DequantizeRow            src/quant.h:65
//   DotRowQuant / DotRowQuantRef / MatMulBlocked / ActiveKernelName
//                            src/matmul.h:35-64
//   Model::Load              src/model.h:115
//   KvCache                  src/kv_cache.h:35-82
//   ForwardFull / Generate   src/qwen3.h:83-142
//   CounterUniform / FilterToProbs / SampleToken
//                            src/sampler.h:46-65
// Every entry catches C++ exceptions and reports them through
// refd_last_error(), mirroring the reference ABI's convention
// (src/engine.cc:175-191).

#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include "dtypes.h"
#include "kv_cache.h"
#include "matmul.h"
#include "model.h"
#include "quant.h"
#include "qwen3.h"
#include "sampler.h"
#include "threads.h"

namespace {

thread_local std::string g_err;

struct RefModel {
  std::unique_ptr<rpg::Model> model;
  rpg::ForwardScratch scratch;
};

int Fail(const std::exception& e) {
  g_err = e.what();
  return -1;
}

}  // namespace

extern "C" {

const char* refd_last_error(void) { return g_err.c_str(); }

const char* refd_active_kernel(void) { return rpg::ActiveKernelName(); }

float refd_f16_to_f32(uint16_t h) { return rpg::F16ToF32(h); }
uint16_t refd_f32_to_f16(float f) { return rpg::F32ToF16(f); }

int refd_dequantize_row(uint32_t type, const uint8_t* src, int64_t n, float* dst) {
  try {
    rpg::DequantizeRow(type, src, n, dst);
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

// Dispatching dot (AVX2 unless RPGBAR_NO_SIMD was set before load).
int refd_dot_row(uint32_t type, const float* a, const uint8_t* w, int64_t k, float* out) {
  try {
    *out = rpg::DotRowQuant(type, a, w, k);
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

// Scalar reference dot (never dispatched).
int refd_dot_row_ref(uint32_t type, const float* a, const uint8_t* w, int64_t k, float* out) {
  try {
    *out = rpg::DotRowQuantRef(type, a, w, k);
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

// QuantMatrix::MatMulBatch semantics over a raw buffer: blocked kernel when it
// takes the call, per-(t,r) DotRowQuant otherwise.  threads <= 0 = serial.
int refd_matmul(uint32_t type, const uint8_t* w, int64_t rows, int64_t cols, const float* X,
                int64_t n, float* OUT, int threads) {
  try {
    std::unique_ptr<rpg::ThreadPool> pool;
    if (threads > 1) pool = std::make_unique<rpg::ThreadPool>(threads);
    rpg::QuantMatrix m(w, type, rows, cols);
    m.MatMulBatch(X, n, OUT, pool.get());
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

float refd_counter_uniform(uint64_t seed, uint64_t counter) {
  return rpg::CounterUniform(seed, counter);
}

uint64_t refd_splitmix64(uint64_t x) { return rpg::SplitMix64(x); }

int refd_filter_to_probs(const float* logits, int64_t n, float temperature, int32_t top_k,
                         float top_p, float* probs) {
  try {
    rpg::SampleOptions o;
    o.temperature = temperature;
    o.top_k = top_k;
    o.top_p = top_p;
    std::vector<float> p;
    rpg::FilterToProbs(logits, n, o, &p);
    std::memcpy(probs, p.data(), p.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int32_t refd_sample_token(const float* logits, int64_t n, float temperature, int32_t top_k,
                          float top_p, float u) {
  rpg::SampleOptions o;
  o.temperature = temperature;
  o.top_k = top_k;
  o.top_p = top_p;
  return rpg::SampleToken(logits, n, o, u);
}

void* refd_model_load(const char* path, int threads, int32_t max_pos) {
  try {
    auto* m = new RefModel();
    m->model = std::make_unique<rpg::Model>(rpg::Model::Load(path, threads, max_pos));
    return m;
  } catch (const std::exception& e) {
    Fail(e);
    return nullptr;
  }
}

void refd_model_free(void* h) { delete static_cast<RefModel*>(h); }

// out: n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab,
// context_length, rope positions, tied(0/1)
int refd_model_config(void* h, int64_t* out) {
  auto* m = static_cast<RefModel*>(h);
  const rpg::ModelConfig& c = m->model->config();
  out[0] = c.n_layers;
  out[1] = c.hidden;
  out[2] = c.n_heads;
  out[3] = c.n_kv_heads;
  out[4] = c.head_dim;
  out[5] = c.intermediate;
  out[6] = c.vocab;
  out[7] = c.context_length;
  out[8] = m->model->rope_positions();
  out[9] = c.tied_embeddings ? 1 : 0;
  return 0;
}

// Copies the model's RoPE table ([positions][hd/2 cos | hd/2 sin]).
int refd_model_rope(void* h, float* out, int64_t max_floats) {
  auto* m = static_cast<RefModel*>(h);
  const rpg::ModelConfig& c = m->model->config();
  const int64_t n = m->model->rope_positions() * c.head_dim;
  if (n > max_floats) return -1;
  std::memcpy(out, m->model->rope_cos(0), static_cast<size_t>(n) * sizeof(float));
  return 0;
}

void* refd_kv_create(void* h, int64_t max_seq) {
  try {
    auto* m = static_cast<RefModel*>(h);
    return new rpg::KvCache(m->model->config(), max_seq);
  } catch (const std::exception& e) {
    Fail(e);
    return nullptr;
  }
}

void refd_kv_free(void* kv) { delete static_cast<rpg::KvCache*>(kv); }
int64_t refd_kv_len(void* kv) { return static_cast<rpg::KvCache*>(kv)->len(); }
int refd_kv_set_len(void* kv, int64_t n) {
  try {
    static_cast<rpg::KvCache*>(kv)->SetLen(n);
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

// ForwardFull; kv may be null.  logits receives seq*vocab floats.
int refd_forward(void* h, void* kv, const int32_t* ids, int64_t seq, float* logits) {
  try {
    auto* m = static_cast<RefModel*>(h);
    std::vector<float> out;
    rpg::ForwardFull(*m->model, ids, seq, &m->scratch, &out, rpg::ForwardOptions(),
                     static_cast<rpg::KvCache*>(kv));
    std::memcpy(logits, out.data(), out.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

// Generate with explicit sampling options; out needs max_tokens slots.
int refd_generate(void* h, void* kv, const float* first_logits, int32_t max_tokens,
                  const int32_t* stop_ids, int32_t n_stop, float temperature, int32_t top_k,
                  float top_p, uint64_t seed, int32_t* out, int32_t* n_out) {
  try {
    auto* m = static_cast<RefModel*>(h);
    rpg::GenerateOptions o;
    o.max_tokens = max_tokens;
    o.stop_ids.assign(stop_ids, stop_ids + n_stop);
    o.sample.temperature = temperature;
    o.sample.top_k = top_k;
    o.sample.top_p = top_p;
    o.seed = seed;
    std::vector<int32_t> gen;
    rpg::Generate(*m->model, static_cast<rpg::KvCache*>(kv), &m->scratch, first_logits, o,
                  &gen);
    std::memcpy(out, gen.data(), gen.size() * sizeof(int32_t));
    *n_out = static_cast<int32_t>(gen.size());
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

}  // extern "C"
