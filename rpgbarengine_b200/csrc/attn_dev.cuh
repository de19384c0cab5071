// attn_dev.cuh -- device building blocks of decode attention shared by the
// per-launch decode kernel (k_attn.cu) and the persistent decode-step kernel
// (k_step.cu): QK-norm + RoPE of a 128-wide head held as a float4 per lane,
// and the transpose-reduction that leaves lane l with the warp-wide sum of
// value l.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace rpgc {
namespace attn {

constexpr float kNegBig = -3.0e38f;

// QK-norm + RoPE of one 128-wide head held as a float4 per lane (dims
// 4*lane..4*lane+3): RMSNorm with a double sum of squares, then the half-split
// rotation with the reference's separate roundings.  The partner dims
// (i +- 64) come from lane^16.
__device__ __forceinline__ float4 norm_rope_head(float4 v, const float* w, const float* cs,
                                                 float eps, int lane) {
  double ss = (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  ss = warp_sum(ss);
  const float scale = (float)(1.0 / sqrt(ss / 128.0 + (double)eps));
  const float4 g = *reinterpret_cast<const float4*>(w + 4 * lane);
  float y[4] = {v.x * scale * g.x, v.y * scale * g.y, v.z * scale * g.z, v.w * scale * g.w};
  float o[4];
  const bool lo = lane < 16;  // dims < 64
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[k], 16);
    const int i = (4 * lane + k) & 63;
    const float c = cs[i], sn = cs[64 + i];
    o[k] = lo ? __fsub_rn(__fmul_rn(y[k], c), __fmul_rn(partner, sn))
              : __fadd_rn(__fmul_rn(y[k], c), __fmul_rn(partner, sn));
  }
  return make_float4(o[0], o[1], o[2], o[3]);
}

// The same with the gains g and the lane's cosines c and sines sn (dims
// (4 lane + k) & 63) already in registers.
__device__ __forceinline__ float4 norm_rope_head_pre(float4 v, float4 g, float4 c, float4 sn, float eps,
                                                     int lane) {
  double ss = (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  ss = warp_sum(ss);
  const float scale = (float)(1.0 / sqrt(ss / 128.0 + (double)eps));
  const float y[4] = {v.x * scale * g.x, v.y * scale * g.y, v.z * scale * g.z, v.w * scale * g.w};
  const float cc[4] = {c.x, c.y, c.z, c.w}, ss4[4] = {sn.x, sn.y, sn.z, sn.w};
  float o[4];
  const bool lo = lane < 16;  // dims < 64
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[k], 16);
    o[k] = lo ? __fsub_rn(__fmul_rn(y[k], cc[k]), __fmul_rn(partner, ss4[k]))
              : __fadd_rn(__fmul_rn(y[k], cc[k]), __fmul_rn(partner, ss4[k]));
  }
  return make_float4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}

// 32 values per lane -> lane l holds the warp-wide sum of value l.
__device__ __forceinline__ float transpose_reduce(float* v, int lane) {
#pragma unroll
  for (int n = 16; n >= 1; n >>= 1) {
    const bool up = (lane & n) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = up ? v[i] : v[i + n];
      const float keep = up ? v[i + n] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, n);
    }
  }
  return v[0];
}

}  // namespace attn
}  // namespace rpgc
