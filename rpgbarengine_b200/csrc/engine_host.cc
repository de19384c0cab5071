// engine_host.cc -- the token-level engine: the reference's per-session
// orchestration of a chat turn (rpg_engine_session_create / _reset /
// _destroy / _generate, src/engine.cc:259-515) over the rpgc token loop.
//
// The host keeps the text side -- chat template, tokenizer, tool-call parser,
// JSON -- and passes each turn's whole rendered prompt as token ids; it gets
// the completion back as token ids.  What the reference does between those
// two points is here, in the same order:
//
//   1. longest common prefix of the prompt with the ids the cache holds
//      (src/engine.cc:383-392); a prompt the cache holds entirely backs off
//      one position so that one row is forwarded (:394-395);
//   2. max_tokens, temperature (clamped to [0, 2]) and seed from the request,
//      else the session's defaults (:399-411);
//   3. every check that can fail before the cache is touched: prompt +
//      max_tokens + 4 must fit the session (:414-419);
//   4. the cache cut back to the prefix, the rest of the prompt forwarded;
//      a forward that fails resets the cache and the cached ids (:422-448);
//   5. stop ids: the model's end-of-sequence id, <|im_end|>, the request's and
//      the session's single-token stop ids (:451-456); sampling with top_k 0
//      and top_p 0.95 (:463-467); the generated ids appended to the cached
//      ids (:470-471);
//   6. the finish reason by tokens (:477-487): "length" when max_tokens ids
//      came and the last is not a stop id, else "stop".  "tool_calls" and
//      the "length" of a completion cut inside a tool call or a think block
//      come from the host's parser, which sees the text.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/rpgc.h"

namespace rpgc {
void set_last_error(const char* msg);  // engine.cu
}  // namespace rpgc

namespace {

constexpr int32_t kDefaultMaxTokens = 256;  // src/engine.cc:43
constexpr int64_t kSeqMargin = 4;           // src/engine.cc:44
constexpr int32_t kDefaultTopK = 0;         // src/engine.cc:46
constexpr float kDefaultTopP = 0.95f;       // src/engine.cc:47
constexpr float kMaxTemperature = 2.0f;     // src/engine.cc:48

struct EngineSession {
  int32_t model = 0;
  int32_t session = 0;  // the rpgc session that owns the KV cache
  int32_t max_seq = 0;
  std::vector<int32_t> cached_ids;  // the ids whose K/V the cache holds, in order
  int32_t max_tokens = kDefaultMaxTokens;
  float temperature = 0.0f;
  uint64_t seed = 0;
  std::vector<int32_t> stop;  // the session's stop ids
  std::mutex mu;              // one generate at a time per session
};

std::mutex g_mu;
std::unordered_map<int32_t, std::unique_ptr<EngineSession>> g_sessions;
int32_t g_next = 1;

struct Failure {
  int code;
  std::string msg;
};

[[noreturn]] void fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw Failure{code, buf};
}

// A failed rpgc call, with its own message.
[[noreturn]] void fail_rc(int rc, const char* what) {
  throw Failure{rc, std::string(what) + ": " + rpgc_last_error()};
}

template <typename F>
int guard(F&& f) {
  try {
    rpgc::set_last_error("");
    return f();
  } catch (const Failure& e) {
    rpgc::set_last_error(e.msg.c_str());
    return e.code;
  } catch (const std::exception& e) {
    rpgc::set_last_error(e.what());
    return RPGC_E_CUDA;
  } catch (...) {
    rpgc::set_last_error("unknown exception");
    return RPGC_E_CUDA;
  }
}

EngineSession* require(int32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  const auto it = g_sessions.find(h);
  if (it == g_sessions.end()) fail(RPGC_E_STATE, "invalid engine session handle %d (destroyed?)", h);
  return it->second.get();
}

float clamp_temperature(float t) {
  if (!(t > 0.0f)) return 0.0f;  // negative and NaN: greedy
  return t > kMaxTemperature ? kMaxTemperature : t;
}

void check_ids(const int32_t* ids, int32_t n, int32_t vocab, const char* what) {
  if (n < 0 || (n > 0 && !ids)) fail(RPGC_E_ARG, "%s: %d ids at NULL", what, n);
  for (int32_t i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= vocab) fail(RPGC_E_ARG, "%s: id %d outside the vocabulary (%d)", what, ids[i], vocab);
}

void add_stop(std::vector<int32_t>* v, int32_t id) {
  if (id >= 0 && std::find(v->begin(), v->end(), id) == v->end()) v->push_back(id);
}

}  // namespace

extern "C" {

int32_t rpgc_engine_session_create(int32_t model, const rpgc_engine_session_opts* opts) {
  int32_t handle = -1;
  const int rc = guard([&] {
    rpgc_model_config c{};
    const int r = rpgc_model_get_config(model, &c);
    if (r != RPGC_OK) fail_rc(r, "engine session");
    const rpgc_engine_session_opts o = opts ? *opts : rpgc_engine_session_opts{};
    const int32_t max_pos = c.max_pos;  // positions of the RoPE table: min(max_pos, context_length)
    const int32_t max_seq = o.max_seq == 0 ? max_pos : o.max_seq;
    if (max_seq <= 0 || max_seq > max_pos) fail(RPGC_E_ARG, "max_seq=%d must be in (0, %d]", max_seq, max_pos);
    int32_t max_tokens = o.max_tokens == 0 ? kDefaultMaxTokens : o.max_tokens;
    if (max_tokens <= 0) fail(RPGC_E_ARG, "max_tokens must be positive (got %d)", max_tokens);
    if (max_tokens >= max_seq) max_tokens = max_seq - 1;  // room for the output (src/engine.cc:281-286)
    check_ids(o.stop_ids, o.n_stop, c.vocab, "session stop ids");
    auto s = std::make_unique<EngineSession>();
    s->model = model;
    s->max_seq = max_seq;
    s->max_tokens = max_tokens;
    s->temperature = clamp_temperature(o.temperature);
    s->seed = o.seed;
    for (int32_t i = 0; i < o.n_stop; ++i) add_stop(&s->stop, o.stop_ids[i]);
    s->session = rpgc_session_create(model, max_seq);
    if (s->session < 0) fail_rc(s->session, "engine session");
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_next <= 0) {
      rpgc_session_destroy(s->session);
      fail(RPGC_E_STATE, "engine session handles exhausted");
    }
    handle = g_next++;
    g_sessions.emplace(handle, std::move(s));
    return RPGC_OK;
  });
  return rc == RPGC_OK ? handle : rc;
}

int rpgc_engine_session_destroy(int32_t h) {
  return guard([&] {
    std::unique_ptr<EngineSession> s;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      const auto it = g_sessions.find(h);
      if (it == g_sessions.end()) return RPGC_OK;  // unknown handle: no-op (src/engine.cc:312-314)
      s = std::move(it->second);
      g_sessions.erase(it);
    }
    std::lock_guard<std::mutex> lk(s->mu);  // a generate in flight finishes first
    rpgc_session_destroy(s->session);
    return RPGC_OK;
  });
}

int rpgc_engine_session_reset(int32_t h) {
  return guard([&] {
    EngineSession* s = require(h);
    std::lock_guard<std::mutex> lk(s->mu);
    // the length goes to zero, the memory stays (src/engine.cc:341-343)
    const int r = rpgc_session_set_len(s->session, 0);
    if (r != RPGC_OK) fail_rc(r, "engine session reset");
    s->cached_ids.clear();
    return RPGC_OK;
  });
}

int64_t rpgc_engine_session_cached(int32_t h, int32_t* ids, int64_t cap) {
  int64_t n = 0;
  const int rc = guard([&] {
    EngineSession* s = require(h);
    std::lock_guard<std::mutex> lk(s->mu);
    n = (int64_t)s->cached_ids.size();
    if (ids && cap > 0) std::copy_n(s->cached_ids.begin(), std::min(n, cap), ids);
    return RPGC_OK;
  });
  return rc == RPGC_OK ? n : rc;
}

int rpgc_engine_generate(int32_t h, const int32_t* ids, int64_t n, const rpgc_engine_request* req,
                         int32_t* out_ids, int32_t out_cap, rpgc_engine_result* res) {
  return guard([&] {
    if (!res || !out_ids) fail(RPGC_E_ARG, "null output");
    *res = rpgc_engine_result{};
    EngineSession* s = require(h);
    std::lock_guard<std::mutex> lk(s->mu);
    rpgc_model_config c{};
    int r = rpgc_model_get_config(s->model, &c);
    if (r != RPGC_OK) fail_rc(r, "engine generate");
    if (!ids || n <= 0) fail(RPGC_E_ARG, "the prompt is empty");  // src/engine.cc:378
    // prompt ids are checked by the forward, as the reference's ForwardFull
    // checks them (src/qwen3.cc:253-254): an id outside the vocabulary is a
    // failed forward, which resets the cache

    // 1. the longest common prefix with the cache (src/engine.cc:383-397)
    const int64_t cached = (int64_t)s->cached_ids.size();
    const int64_t kv_len = rpgc_session_len(s->session);
    if (kv_len < 0) fail_rc((int)kv_len, "engine generate");
    if (kv_len != cached)
      fail(RPGC_E_STATE, "internal state: %lld cached ids but the cache holds %lld positions", (long long)cached,
           (long long)kv_len);
    int64_t lcp = 0;
    while (lcp < cached && lcp < n && s->cached_ids[(size_t)lcp] == ids[lcp]) ++lcp;
    if (lcp == n) lcp = n - 1;  // forward at least one row
    const int64_t rows = n - lcp;

    // 2. options: the request's, else the session's (src/engine.cc:399-411)
    int32_t max_tokens = req && req->max_tokens > 0 ? req->max_tokens : s->max_tokens;
    const float temperature = clamp_temperature(req && req->set_temperature ? req->temperature : s->temperature);
    const uint64_t seed = req && req->set_seed ? req->seed : s->seed;
    std::vector<int32_t> stop;
    {
      int32_t eos = -1, im_end = -1;
      r = rpgc_model_special_ids(s->model, &eos, &im_end);
      if (r != RPGC_OK) fail_rc(r, "engine generate");
      add_stop(&stop, eos);
      add_stop(&stop, im_end);
    }
    if (req) check_ids(req->stop_ids, req->n_stop, c.vocab, "request stop ids");
    if (req)
      for (int32_t i = 0; i < req->n_stop; ++i) add_stop(&stop, req->stop_ids[i]);
    for (int32_t id : s->stop) add_stop(&stop, id);

    // 3. every check that can fail comes before the cache is touched
    //    (src/engine.cc:412-419)
    if (n + max_tokens + kSeqMargin > s->max_seq)
      fail(RPGC_E_CONTEXT_FULL,
           "sequence too long: prompt %lld + max_tokens %d + margin %lld exceeds the session's %d positions "
           "(a larger max_seq, or reset the session)",
           (long long)n, max_tokens, (long long)kSeqMargin, s->max_seq);
    if (max_tokens > out_cap) fail(RPGC_E_ARG, "out_ids holds %d ids, max_tokens is %d", out_cap, max_tokens);
    if ((int)stop.size() > RPGC_MAX_STOP) fail(RPGC_E_ARG, "%zu stop ids, at most %d", stop.size(), RPGC_MAX_STOP);

    // 4. prefill of what the cache does not hold (src/engine.cc:421-448)
    auto reset = [&] {
      rpgc_session_set_len(s->session, 0);
      s->cached_ids.clear();
    };
    r = rpgc_session_set_len(s->session, lcp);
    if (r == RPGC_OK) r = rpgc_forward(s->session, ids + lcp, rows, nullptr, nullptr);
    if (r != RPGC_OK) {
      const std::string msg = std::string("engine generate: forward: ") + rpgc_last_error();
      reset();  // a cache of uncertain length is not reused
      throw Failure{r, msg};
    }
    s->cached_ids.assign(ids, ids + n);

    // 5. generation (src/engine.cc:450-471)
    rpgc_gen_opts o{};
    o.max_tokens = max_tokens;
    o.stop_ids = stop.data();
    o.n_stop = (int32_t)stop.size();
    o.temperature = temperature;
    o.top_k = kDefaultTopK;
    o.top_p = kDefaultTopP;
    o.seed = seed;
    int32_t n_out = 0;
    r = rpgc_generate(s->session, &o, out_ids, &n_out);
    if (r != RPGC_OK) {
      const std::string msg = std::string("engine generate: ") + rpgc_last_error();
      // a failed decode leaves the cache at the prompt; anything else is reset
      if (rpgc_session_len(s->session) != n) reset();
      throw Failure{r, msg};
    }
    s->cached_ids.insert(s->cached_ids.end(), out_ids, out_ids + n_out);

    // 6. finish reason by tokens (src/engine.cc:477-487)
    const bool stopped = n_out > 0 && std::find(stop.begin(), stop.end(), out_ids[n_out - 1]) != stop.end();
    res->finish = n_out >= max_tokens && !stopped ? RPGC_FINISH_LENGTH : RPGC_FINISH_STOP;
    res->n_out = n_out;
    res->prompt_tokens = n;
    res->reused = lcp;
    return RPGC_OK;
  });
}

}  // extern "C"
