// k_gemm_simt.cu -- prefill matmul over raw ggml blocks on CUDA cores (for
// shapes the tensor-core path does not take: K not a multiple of 64, or no
// scratch), and the dispatch between the two.
//
// Replaces the reference's 8-token blocked kernel (MatMulBlocked,
// src/matmul_avx2.cc:482-507): one dequantised weight tile in shared memory
// serves a tile of 128 tokens.  Weights are dequantised bit-exactly (the
// reference's fp32 values); products are accumulated in fp32.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

constexpr int BM = 64, BN = 128, BK = 32;

__global__ void __launch_bounds__(256) gemm_simt_kernel(uint32_t type, const uint8_t* __restrict__ w,
                                                        int64_t rows, int64_t K, int64_t row_bytes,
                                                        const float* __restrict__ X, int64_t n,
                                                        float* __restrict__ out, int64_t ldo,
                                                        int accumulate) {
  __shared__ __align__(16) float Ws[BK][BM + 4];
  __shared__ __align__(16) float Xs[BK][BN + 4];
  const int tid = threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.x * BM, t0 = (int64_t)blockIdx.y * BN;
  const int ty = tid >> 4, tx = tid & 15;  // rows ty*4.., tokens tx*8..
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    {  // weights: 64 rows x 32 elements, 8 per thread
      const int r = tid >> 2, kk = (tid & 3) * 8;
      const int64_t gr = r0 + r;
      if (gr < rows) {
        const uint8_t* row = w + gr * row_bytes;
#pragma unroll
        for (int j = 0; j < 8; ++j) Ws[kk + j][r] = deq_elem(type, row, k0 + kk + j);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) Ws[kk + j][r] = 0.0f;
      }
    }
    {  // activations: 128 tokens x 32, 16 per thread
      const int t = tid >> 1, kk = (tid & 1) * 16;
      const int64_t gt = t0 + t;
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gt < n) v = *reinterpret_cast<const float4*>(X + gt * K + k0 + kk + j);
        Xs[kk + j + 0][t] = v.x;
        Xs[kk + j + 1][t] = v.y;
        Xs[kk + j + 2][t] = v.z;
        Xs[kk + j + 3][t] = v.w;
      }
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < BK; ++k) {
      const float4 wv = *reinterpret_cast<const float4*>(&Ws[k][ty * 4]);
      const float4 xa = *reinterpret_cast<const float4*>(&Xs[k][tx * 8]);
      const float4 xb = *reinterpret_cast<const float4*>(&Xs[k][tx * 8 + 4]);
      const float wr[4] = {wv.x, wv.y, wv.z, wv.w};
      const float xr[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(wr[i], xr[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + ty * 4 + i;
    if (r >= rows) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t t = t0 + tx * 8 + j;
      if (t >= n) continue;
      float* o = out + t * ldo + r;
      *o = accumulate ? *o + acc[i][j] : acc[i][j];
    }
  }
}

}  // namespace

size_t gemm_scratch_bytes(int64_t n, int64_t K) { return gemm_tc_scratch_bytes(n, K); }

bool gemm_uses_tc(uint32_t type, int64_t n, int64_t K, size_t scratch_bytes) {
  return scratch_bytes >= gemm_tc_scratch_bytes(n, K) && gemm_tc_supported(type, K);
}

cudaError_t gemm_launch(uint32_t type, const uint8_t* w, int64_t rows, int64_t K,
                        int64_t row_bytes, const float* X, int64_t n, float* out, int64_t ldo,
                        bool accumulate, void* scratch, size_t scratch_bytes, cudaStream_t s,
                        bool x_split_ready, const float* glu) {
  if (scratch && gemm_uses_tc(type, n, K, scratch_bytes))
    return gemm_tc_launch(type, w, rows, K, row_bytes, X, n, out, ldo, accumulate, scratch,
                          scratch_bytes, s, x_split_ready, glu);
  if (glu) return cudaErrorInvalidValue;  // the fused SwiGLU is a tensor-core epilogue
  if (K % BK != 0 || (reinterpret_cast<uintptr_t>(X) & 15)) return cudaErrorInvalidValue;
  dim3 grid((unsigned)((rows + BM - 1) / BM), (unsigned)((n + BN - 1) / BN));
  gemm_simt_kernel<<<grid, 256, 0, s>>>(type, w, rows, K, row_bytes, X, n, out, ldo,
                                        accumulate ? 1 : 0);
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) count_launches(1);
  return e;
}

}  // namespace rpgc
