// noalloc.cu -- decode attention that allocates nothing.
//
// Some callers cannot allocate device memory at the moment they need a
// result: a host that runs inside another runtime's memory budget (a game
// engine that owns the GPU heap and forbids foreign cudaMalloc/cudaFree), a
// caller on a latency-critical path where an allocation may block or
// synchronise, or code that must not touch the allocator while another
// component holds it.  rpgc_attention_decode allocates its split-K scratch
// per call; this variant uses a fixed scratch array that lives in the module
// image instead, so a call performs no allocation at all.
//
// The scratch is a file-scope __device__ array of kScratchBytes (2.03 MiB),
// present on every GPU that loads the library until the process exits.  It
// holds the per-kv-head completion counters (first 256 bytes, which each call
// clears) and the split partial results.  All calls share it: calls whose
// kernels overlap on the GPU (different streams, or different host threads)
// race on it and must be serialised by the caller.
#include <cuda_runtime.h>

#include <climits>
#include <mutex>
#include <string>

#include "../../include/rpgc.h"
#include "kernels.h"

namespace rpgc {
void set_last_error(const char* msg);  // engine.cu
namespace {

constexpr int kSplits = 32;       // split-K factor over positions
constexpr int kMaxKvHeads = 16;   // largest n_kv_heads accepted
constexpr int kMaxGroupNA = 8;    // largest n_heads / n_kv_heads accepted
constexpr size_t kCounterBytes = 256;
constexpr size_t kPartialFloats = (size_t)kMaxKvHeads * kSplits * kMaxGroupNA * 130;
constexpr size_t kScratchBytes = kCounterBytes + kPartialFloats * sizeof(float);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};


// Device address of the scratch array on the current device, looked up once
// per device (the host-side symbol is only a stand-in and must never be
// handed to a kernel).
cudaError_t scratch_for_current_device(unsigned char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
  return cudaSuccess;
}

}  // namespace
}  // namespace rpgc

extern "C" int rpgc_attention_decode_noalloc(const float* q, const float* k_cache,
                                             const float* v_cache, int64_t max_seq,
                                             int32_t n_heads, int32_t n_kv_heads,
                                             int32_t head_dim, int64_t pos, float* out,
                                             void* stream) {
  using namespace rpgc;
  set_last_error("");
  if (!q || !k_cache || !v_cache || !out || n_heads <= 0 || n_kv_heads <= 0 || max_seq <= 0) {
    set_last_error("attention_decode_noalloc: null pointer or non-positive size");
    return RPGC_E_ARG;
  }
  if (head_dim != 128 || n_heads % n_kv_heads) {
    set_last_error("attention_decode_noalloc: head_dim must be 128 and n_heads a multiple of "
                   "n_kv_heads");
    return RPGC_E_ARG;
  }
  if (n_kv_heads > kMaxKvHeads || n_heads / n_kv_heads > kMaxGroupNA) {
    set_last_error("attention_decode_noalloc: shape exceeds the fixed scratch "
                   "(at most 16 kv heads and 8 query heads per kv head)");
    return RPGC_E_ARG;
  }
  if (pos < 0 || pos >= max_seq || pos > INT32_MAX - 1) {
    set_last_error("attention_decode_noalloc: pos out of range");
    return RPGC_E_ARG;
  }
  unsigned char* base = nullptr;
  cudaError_t e = scratch_for_current_device(&base);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RPGC_E_CUDA;
  }
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  int32_t* counters = reinterpret_cast<int32_t*>(base);
  // The completion counters must start at zero.
  e = cudaMemsetAsync(counters, 0, n_kv_heads * sizeof(int32_t), cs);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RPGC_E_CUDA;
  }
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
  a.partial = reinterpret_cast<float*>(base + kCounterBytes);
  a.counters = counters;
  a.max_splits = kSplits;
  e = attn_decode_launch(a, cs);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RPGC_E_CUDA;
  }
  return RPGC_OK;
}
