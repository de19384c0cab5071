// noalloc.cu -- the prefill matmul without any allocation.
//
// rpgc_matmul gives its tensor-core kernels scratch memory that it allocates
// for the call (stream-ordered cudaMallocAsync): the fp16 hi/lo split of the
// input rows, one scale per row, and the split-K partial sums.  Some callers
// cannot let the library allocate device memory: a game engine or another
// runtime that owns the GPU heap and forbids foreign cudaMalloc/cudaFree, or a
// caller on a path where an allocation may block, synchronise or fail under
// memory pressure.  rpgc_matmul_noalloc runs the same kernels with that
// scratch in a fixed array of this library instead.
//
// The array is kNoallocScratchBytes (32 MiB) of device memory on every GPU
// that loads the library, held until the process exits.  All calls on a
// device share it and it keeps the last call's contents; every call writes
// all of the scratch it reads before reading it, so nothing has to start at
// zero.  Calls whose work overlaps on the GPU (different streams, or no
// ordering between them) race on the array: order them.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "../../include/rpgc.h"
#include "kernels.h"

namespace rpgc {
void set_last_error(const char* msg);  // engine.cu
}  // namespace rpgc

namespace {

constexpr size_t kNoallocScratchBytes = size_t(32) << 20;

// Device code could name this array directly; host code must not pass its
// name to a kernel (on the host it is only a stand-in for the symbol): it
// takes the device address from cudaGetSymbolAddress, per device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

// The array's address on the current device, looked up on every call with
// that device current.  The lookup is cheap, and an address kept from an
// earlier call could be stale: after cudaDeviceReset, or under another
// driver context on the same ordinal, the module (and the array) is loaded
// again at another address.
cudaError_t scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  *out = p;
  return cudaSuccess;
}

int64_t row_bytes(uint32_t type, int64_t cols) {
  switch (type) {
    case RPGC_F32: return cols * 4;
    case RPGC_Q8_0: return cols % 32 ? -1 : cols / 32 * 34;
    case RPGC_Q4_K: return cols % 256 ? -1 : cols / 256 * 144;
    case RPGC_Q6_K: return cols % 256 ? -1 : cols / 256 * 210;
    default: return -1;
  }
}

int fail_arg(const char* msg) {
  rpgc::set_last_error(msg);
  return RPGC_E_ARG;
}

}  // namespace

extern "C" int rpgc_matmul_noalloc(uint32_t type, const void* w, int64_t rows, int64_t cols,
                                   const float* X, int64_t n, float* OUT, void* stream) {
  using namespace rpgc;
  set_last_error("");
  if (!w || !X || !OUT || rows <= 0 || cols <= 0 || n <= 0)
    return fail_arg("matmul_noalloc: null pointer or non-positive size");
  const int64_t rb = row_bytes(type, cols);
  if (rb < 0 || cols % 32)
    return fail_arg("matmul_noalloc: type must be F32, Q8_0, Q4_K or Q6_K with cols a multiple of "
                    "its block (and of 32)");
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(X)) & 15)
    return fail_arg("matmul_noalloc: w and X must be 16-byte aligned");
  if (n == 1) return rpgc_matvec(type, w, rows, cols, X, OUT, stream);  // the GEMV needs no scratch
  const size_t need = gemm_scratch_bytes(n, cols);
  if (need > kNoallocScratchBytes) {
    char msg[256];
    std::snprintf(msg, sizeof msg,
                  "matmul_noalloc: %lld rows of %lld columns need %zu bytes of scratch; the fixed "
                  "array holds %zu (about 4 n cols + 36864 n bytes are needed): use rpgc_matmul",
                  (long long)n, (long long)cols, need, kNoallocScratchBytes);
    return fail_arg(msg);
  }
  void* scratch = nullptr;
  cudaError_t e = scratch_address(&scratch);
  if (e == cudaSuccess)
    e = gemm_launch(type, static_cast<const uint8_t*>(w), rows, cols, rb, X, n, OUT, rows, false,
                    scratch, kNoallocScratchBytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RPGC_E_CUDA;
  }
  return RPGC_OK;
}
