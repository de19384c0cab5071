// noalloc.cu -- decode attention that allocates nothing.
//
// Some callers cannot allocate device memory at the moment they need a
// result: a host that runs inside another runtime's memory budget (a game
// engine that owns the GPU heap and forbids foreign cudaMalloc/cudaFree), a
// caller on a latency-critical path where an allocation may block or
// synchronise, or code that must not touch the allocator while another
// component holds it.  This entry point guarantees, as part of its contract,
// that a call performs no allocation and holds no state between calls: the
// decode attention kernel merges its position splits inside a thread-block
// cluster (distributed shared memory), so it needs no global scratch, and
// calls on different streams may overlap freely.
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "../../include/rpgc.h"
#include "kernels.h"

namespace rpgc {
void set_last_error(const char* msg);  // engine.cu
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
  const int32_t grp = n_heads / n_kv_heads;
  if (!(grp == 1 || grp == 2 || grp == 4 || grp == 8)) {
    set_last_error("attention_decode_noalloc: GQA group (n_heads / n_kv_heads) must be 1, 2, 4 or 8");
    return RPGC_E_ARG;
  }
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) {
    set_last_error("attention_decode_noalloc: caches must be 16-byte aligned");
    return RPGC_E_ARG;
  }
  if (pos < 0 || pos >= max_seq || pos > INT32_MAX - 1) {
    set_last_error("attention_decode_noalloc: pos out of range");
    return RPGC_E_ARG;
  }
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
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
  const cudaError_t e = attn_decode_launch(a, cs);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RPGC_E_CUDA;
  }
  return RPGC_OK;
}
