// k_misc.cu -- dequantisation, embedding gather, row RMSNorm, SwiGLU, step
// bookkeeping.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

// DequantizeRow over a row-major matrix (src/quant.cc:416-436), bit-exact.
__global__ void dequant_kernel(uint32_t type, const uint8_t* __restrict__ w, int64_t rows,
                               int64_t cols, int64_t row_bytes, float* __restrict__ out) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, e = i - r * cols;
    out[i] = deq_elem(type, w + r * row_bytes, e);
  }
}

// Embedding lookup = dequantise one row per token (QuantMatrix::Row,
// src/model.cc:32-37).
__global__ void embed_kernel(uint32_t type, const uint8_t* __restrict__ embd, int64_t row_bytes,
                             int64_t n_rows, int32_t hidden, const int32_t* __restrict__ ids,
                             float* __restrict__ x, const DecodeState* st, int32_t* err) {
  grid_dep_wait();
  if (st && !st->active) return;
  const int64_t t = blockIdx.y;
  const int32_t id = st ? st->token : ids[t];
  if (id < 0 || (int64_t)id >= n_rows) {  // device-resident ids never passed a host check
    if (err && blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, kErrBadToken);
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < hidden; e += gridDim.x * blockDim.x)
      x[t * hidden + e] = 0.0f;
    return;
  }
  const uint8_t* row = embd + (int64_t)id * row_bytes;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < hidden; e += gridDim.x * blockDim.x)
    x[t * hidden + e] = deq_elem(type, row, e);
}

// out[t] = RmsNorm(x[t], w) (src/kernels.h:56-63): double sum of squares,
// float scale, (x*scale)*w.
__global__ void rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                    int32_t dim, float eps, float* __restrict__ out) {
  __shared__ double red[32];
  const int64_t t = blockIdx.x;
  const float* xr = x + t * dim;
  double ss = 0.0;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float v = xr[i];
    ss += (double)v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  double tot = 0.0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float scale = (float)(1.0 / sqrt(tot / (double)dim + (double)eps));
  for (int i = threadIdx.x; i < dim; i += blockDim.x) out[t * dim + i] = xr[i] * scale * w[i];
}

// gate = silu(gate) * up (src/kernels.h:82-92).
__global__ void swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = g[i];
    g[i] = (v / (1.0f + expf(-v))) * u[i];
  }
}

__global__ void state_set_kernel(DecodeState* st, const DecodeState v) {
  grid_dep_wait();
  *st = v;
}

__global__ void advance_kernel(DecodeState* st) {
  grid_dep_wait();
  if (st->active) st->pos += 1;
}

}  // namespace

cudaError_t dequant_launch(uint32_t type, const uint8_t* w, int64_t rows, int64_t cols,
                           int64_t row_bytes, float* out, cudaStream_t s) {
  const int64_t total = rows * cols;
  if (total <= 0) return cudaSuccess;
  const int64_t nb_ = (total + 255) / 256;
  const int blocks = (int)(nb_ < 148 * 16 ? nb_ : 148 * 16);
  dequant_kernel<<<blocks, 256, 0, s>>>(type, w, rows, cols, row_bytes, out);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

cudaError_t embed_launch(uint32_t type, const uint8_t* embd, int64_t row_bytes, int64_t n_rows,
                         int32_t hidden, const int32_t* ids, int64_t n, float* x,
                         const DecodeState* st, int32_t* err, cudaStream_t s) {
  dim3 grid((hidden + 255) / 256, (unsigned)n);
  embed_kernel<<<grid, 256, 0, s>>>(type, embd, row_bytes, n_rows, hidden, ids, x, st, err);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

// Batched decode: row b of src goes to dst[b] when session b took part in
// this step (its state is active), so a session that has stopped keeps the
// logits of its last real step.
__global__ void commit_rows_kernel(const float* __restrict__ src, int64_t n_cols, float* const* dst,
                                   DecodeState* const* states) {
  const int64_t b = blockIdx.y;
  if (!states[b]->active) return;
  const float* s = src + b * n_cols;
  float* d = dst[b];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_cols; i += (int64_t)gridDim.x * blockDim.x)
    d[i] = s[i];
}

cudaError_t commit_rows_launch(const float* src, int64_t n_cols, float* const* dst, DecodeState* const* states,
                               int32_t n, cudaStream_t s) {
  if (n < 1 || n > 65535 || n_cols <= 0) return cudaErrorInvalidValue;
  commit_rows_kernel<<<dim3(64, (unsigned)n), 256, 0, s>>>(src, n_cols, dst, states);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

// Batched decode: how many of the n sessions are still active (one block).
__global__ void count_active_kernel(DecodeState* const* states, int32_t n, int32_t* out) {
  int c = 0;
  for (int32_t b = threadIdx.x; b < n; b += blockDim.x) c += states[b]->active ? 1 : 0;
  c = __reduce_add_sync(0xffffffffu, c);
  __shared__ int part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    *out = t;
  }
}

cudaError_t count_active_launch(DecodeState* const* states, int32_t n, int32_t* out, cudaStream_t s) {
  if (n < 1) return cudaErrorInvalidValue;
  count_active_kernel<<<1, 256, 0, s>>>(states, n, out);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

cudaError_t rmsnorm_rows_launch(const float* x, const float* w, int64_t n, int32_t dim, float eps,
                                float* out, cudaStream_t s) {
  rmsnorm_rows_kernel<<<(unsigned)n, 256, 0, s>>>(x, w, dim, eps, out);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

cudaError_t swiglu_launch(float* gate, const float* up, int64_t count, cudaStream_t s) {
  const int64_t nb_ = (count + 255) / 256;
  const int blocks = (int)(nb_ < 148 * 16 ? nb_ : 148 * 16);
  swiglu_kernel<<<blocks, 256, 0, s>>>(gate, up, count);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

cudaError_t state_set_launch(DecodeState* st, const DecodeState& v, cudaStream_t s) {
  state_set_kernel<<<1, 1, 0, s>>>(st, v);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

cudaError_t advance_launch(DecodeState* st, cudaStream_t s) {
  advance_kernel<<<1, 1, 0, s>>>(st);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

// dst[t][r * vl + j] = src[r][t][j]: the ranks' vocabulary slices of nc
// rows of logits, gathered rank-major, interleaved back into rows.
__global__ void gather_vocab_kernel(const float* __restrict__ src, int world, int64_t nc, int64_t vl,
                                    float* __restrict__ dst) {
  const int64_t total = (int64_t)world * nc * vl;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (nc * vl), rem = i - r * nc * vl, t = rem / vl, j = rem - t * vl;
    dst[t * world * vl + r * vl + j] = src[i];
  }
}

cudaError_t gather_vocab_launch(const float* src, int world, int64_t nc, int64_t vl, float* dst,
                                cudaStream_t s) {
  const int64_t total = (int64_t)world * nc * vl;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  gather_vocab_kernel<<<blocks, 256, 0, s>>>(src, world, nc, vl, dst);
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

}  // namespace rpgc
