// k_attn.cu -- QK-norm + RoPE + KV-cache write, and GQA attention over the
// device KV cache (decode: split-K flash-decode; prefill: tiled causal).
//
// Reference: QK-norm before RoPE (src/qwen3.cc:141-152), half-split RoPE
// (src/kernels.h:108-120), cache layout ((l*nkv + h)*max_seq + pos)*hd
// (src/kv_cache.cc:29-33), AttentionFromCache with a softmax over [0, pos]
// (src/qwen3.cc:79-117).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

constexpr float kNegBig = -3.0e38f;

// One block per (token, head); hd threads.  q heads first, then kv heads.
__global__ void qkv_rope_kernel(const QkvArgs a) {
  grid_dep_wait();
  const DecodeState* st = a.state;
  if (st && !st->active) return;
  __shared__ double red[8];
  __shared__ float y[256];
  const int64_t t = blockIdx.x;
  const int h = blockIdx.y, i = threadIdx.x, hd = a.hd, half = hd >> 1;
  const int64_t pos = st ? (int64_t)st->pos : a.pos0 + t;
  const bool isq = h < a.n_heads;
  const int kh = h - a.n_heads;
  const float* src = isq ? a.q + (t * a.n_heads + h) * hd : a.k + (t * a.n_kv + kh) * hd;
  const float x = src[i];
  double ss = warp_sum((double)x * x);
  if ((i & 31) == 0) red[i >> 5] = ss;
  __syncthreads();
  double tot = 0.0;
  for (int w = 0; w < (hd + 31) / 32; ++w) tot += red[w];
  const float scale = (float)(1.0 / sqrt(tot / (double)hd + (double)a.eps));
  y[i] = x * scale * (isq ? a.q_norm : a.k_norm)[i];
  __syncthreads();
  const float* cs = a.rope + pos * hd;  // hd/2 cos then hd/2 sin
  float o;
  if (i < half) {
    o = __fsub_rn(__fmul_rn(y[i], cs[i]), __fmul_rn(y[i + half], cs[half + i]));
  } else {
    const int j = i - half;
    o = __fadd_rn(__fmul_rn(y[i], cs[j]), __fmul_rn(y[j], cs[half + j]));
  }
  if (isq) {
    a.q[(t * a.n_heads + h) * hd + i] = o;
  } else {
    const int64_t off = ((int64_t)kh * a.max_seq + pos) * hd + i;
    a.kc[off] = o;
    a.vc[off] = a.v[(t * a.n_kv + kh) * hd + i];
  }
}

// ---------------------------------------------------------------- decode
// grid (n_kv, splits), 128 threads.  hd == 128 (4 dims per lane), group <= 8.
constexpr int kMaxGroup = 8;
constexpr int kPre = 4;  // positions per warp whose K/V are loaded up front

// QK-norm + RoPE of one 128-wide head held as a float4 per lane (dims
// 4*lane..4*lane+3): RMSNorm with a double sum of squares, then the half-split
// rotation with the reference's separate roundings.  `mine` is this lane's
// float4; the partner dims (i +- 64) come from lane^16.
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

__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnArgs a) {
  grid_dep_wait();
  const DecodeState* st = a.state;
  if (st && !st->active) return;
  __shared__ __align__(16) float sm[4][kMaxGroup][132];  // rows padded to 16 B
  __shared__ __align__(16) float4 knew_s[32], vnew_s[32];
  __shared__ float fsc[kMaxGroup][32];
  __shared__ int s_last;
  const int kh = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.n_heads / a.n_kv, hd = a.hd;
  const int pos = st ? st->pos : (int)a.pos0;
  const int L = pos + 1;  // keys [0, pos]
  const int chunk = (L + S - 1) / S;
  const int c0 = split * chunk, c1 = min(L, c0 + chunk);
  const float scale = 1.0f / sqrtf((float)hd);
  const float* kb = a.kc + (int64_t)kh * a.max_seq * hd;
  const float* vb = a.vc + (int64_t)kh * a.max_seq * hd;
  const bool fused = a.q_norm != nullptr;
  const bool has_new = fused && c0 <= pos && pos < c1;  // this split owns the new token
  const float* cs = fused ? a.rope + (int64_t)pos * hd : nullptr;

  float4 qv[kMaxGroup], ov[kMaxGroup];
  float m[kMaxGroup], l[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g < G) {
      qv[g] = *reinterpret_cast<const float4*>(a.q + (kh * G + g) * hd + 4 * lane);
      if (fused) qv[g] = norm_rope_head(qv[g], a.q_norm, cs, a.eps, lane);
    }
    ov[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    m[g] = kNegBig;
    l[g] = 0.0f;
  }
  if (has_new && warp == 0) {
    // the new token's k/v: normalise + rotate k, write both into the cache
    float4 k4 = *reinterpret_cast<const float4*>(a.k_new + kh * hd + 4 * lane);
    k4 = norm_rope_head(k4, a.k_norm, cs, a.eps, lane);
    const float4 v4 = *reinterpret_cast<const float4*>(a.v_new + kh * hd + 4 * lane);
    const int64_t off = ((int64_t)kh * a.max_seq + pos) * hd + 4 * lane;
    *reinterpret_cast<float4*>(a.kc_w + off) = k4;
    *reinterpret_cast<float4*>(a.vc_w + off) = v4;
    knew_s[lane] = k4;
    vnew_s[lane] = v4;
  }
  __syncthreads();
  // positions of this warp: c0 + warp + 4*i; K/V of up to kPre loaded at once
  for (int p0 = c0 + warp; p0 < c1; p0 += 4 * kPre) {
    float4 kr[kPre], vr[kPre];
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
      const int p = p0 + 4 * i;
      if (p < c1) {
        if (has_new && p == pos) {
          kr[i] = knew_s[lane];
          vr[i] = vnew_s[lane];
        } else {
          kr[i] = *reinterpret_cast<const float4*>(kb + (int64_t)p * hd + 4 * lane);
          vr[i] = *reinterpret_cast<const float4*>(vb + (int64_t)p * hd + 4 * lane);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
      if (p0 + 4 * i >= c1) break;
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g >= G) break;
        float s = qv[g].x * kr[i].x + qv[g].y * kr[i].y + qv[g].z * kr[i].z + qv[g].w * kr[i].w;
        s = warp_sum(s) * scale;
        const float mn = fmaxf(m[g], s);
        const float corr = expf(m[g] - mn), pe = expf(s - mn);
        l[g] = l[g] * corr + pe;
        ov[g].x = ov[g].x * corr + pe * vr[i].x;
        ov[g].y = ov[g].y * corr + pe * vr[i].y;
        ov[g].z = ov[g].z * corr + pe * vr[i].z;
        ov[g].w = ov[g].w * corr + pe * vr[i].w;
        m[g] = mn;
      }
    }
  }
  // merge the 4 warps of this split
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g >= G) break;
    *reinterpret_cast<float4*>(&sm[warp][g][4 * lane]) = ov[g];
    if (lane == 0) {
      sm[warp][g][128] = m[g];
      sm[warp][g][129] = l[g];
    }
  }
  __syncthreads();
  float* part = a.partial + ((int64_t)kh * S + split) * G * 130;
  for (int idx = threadIdx.x; idx < G * 128; idx += 128) {
    const int g = idx >> 7, d = idx & 127;
    float M = kNegBig;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[w][g][128]);
    float O = 0.0f, Lsum = 0.0f;
    for (int w = 0; w < 4; ++w) {
      const float f = expf(sm[w][g][128] - M);
      O += sm[w][g][d] * f;
      Lsum += sm[w][g][129] * f;
    }
    part[g * 130 + d] = O;
    if (d == 0) {
      part[g * 130 + 128] = M;
      part[g * 130 + 129] = Lsum;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&a.counters[kh], 1) == S - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // last split of this kv head: combine all splits (S <= 32: one lane per split)
  const float* pk = a.partial + (int64_t)kh * S * G * 130;
  for (int g = warp; g < G; g += 4) {
    const float ms = lane < S ? __ldcg(pk + (lane * G + g) * 130 + 128) : kNegBig;
    const float ls = lane < S ? __ldcg(pk + (lane * G + g) * 130 + 129) : 0.0f;
    const float M = warp_max(ms);
    const float f = lane < S ? expf(ms - M) : 0.0f;
    const float Lsum = warp_sum(ls * f);
    fsc[g][lane] = f / Lsum;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * 128; idx += 128) {
    const int g = idx >> 7, d = idx & 127;
    float O = 0.0f;
    for (int s = 0; s < S; ++s) O += __ldcg(pk + (s * G + g) * 130 + d) * fsc[g][s];
    a.out[(kh * G + g) * hd + d] = O;
  }
  if (threadIdx.x == 0) a.counters[kh] = 0;
}

// --------------------------------------------------------------- prefill
// grid (n_heads, ceil(n/64)), 256 threads; hd == 128.
constexpr int QT = 64, KT = 64, HD = 128;

__global__ void __launch_bounds__(256) attn_prefill_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float fsm[];
  float* Qs = fsm;             // [HD][QT]
  float* Ks = Qs + HD * QT;    // [HD][KT]
  float* Vs = Ks + HD * KT;    // [KT][HD]
  float* Ps = Vs + KT * HD;    // [KT][QT]
  const int h = blockIdx.x;
  const int64_t qt0 = (int64_t)blockIdx.y * QT;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int G = a.n_heads / a.n_kv, kh = h / G;
  const float scale = 1.0f / sqrtf((float)HD);
  const int64_t qpos0 = a.pos0 + qt0;
  const int64_t nq = min((int64_t)QT, a.n - qt0);
  const int64_t key_end = qpos0 + nq;  // keys [0, key_end)
  const float* kb = a.kc + (int64_t)kh * a.max_seq * HD;
  const float* vb = a.vc + (int64_t)kh * a.max_seq * HD;

  for (int idx = tid; idx < QT * (HD / 4); idx += 256) {
    const int i = idx % QT, c = idx / QT;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < nq) v = *reinterpret_cast<const float4*>(a.q + ((qt0 + i) * a.n_heads + h) * HD + 4 * c);
    Qs[(4 * c + 0) * QT + i] = v.x;
    Qs[(4 * c + 1) * QT + i] = v.y;
    Qs[(4 * c + 2) * QT + i] = v.z;
    Qs[(4 * c + 3) * QT + i] = v.w;
  }
  float m[4], l[4], o[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = kNegBig;
    l[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.0f;
  }
  for (int64_t k0 = 0; k0 < key_end; k0 += KT) {
    __syncthreads();
    for (int idx = tid; idx < KT * (HD / 4); idx += 256) {
      const int j = idx % KT, c = idx / KT;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + j < key_end) kv = *reinterpret_cast<const float4*>(kb + (k0 + j) * HD + 4 * c);
      Ks[(4 * c + 0) * KT + j] = kv.x;
      Ks[(4 * c + 1) * KT + j] = kv.y;
      Ks[(4 * c + 2) * KT + j] = kv.z;
      Ks[(4 * c + 3) * KT + j] = kv.w;
    }
    for (int idx = tid; idx < KT * (HD / 4); idx += 256) {
      const int j = idx / (HD / 4), c = idx % (HD / 4);
      float4 vv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + j < key_end) vv = *reinterpret_cast<const float4*>(vb + (k0 + j) * HD + 4 * c);
      *reinterpret_cast<float4*>(Vs + j * HD + 4 * c) = vv;
    }
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 8
    for (int d = 0; d < HD; ++d) {
      const float4 qv = *reinterpret_cast<const float4*>(Qs + d * QT + ty * 4);
      const float4 kv = *reinterpret_cast<const float4*>(Ks + d * KT + tx * 4);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qa[i], ka[j], s[i][j]);
    }
    float corr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t qp = qpos0 + ty * 4 + i;
      float rmax = kNegBig;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t kp = k0 + tx * 4 + j;
        s[i][j] = (kp <= qp && kp < key_end) ? s[i][j] * scale : -INFINITY;
        rmax = fmaxf(rmax, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
      const float mn = fmaxf(m[i], rmax);
      corr[i] = expf(m[i] - mn);
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = expf(s[i][j] - mn);
        rs += s[i][j];
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * corr[i] + rs;
      m[i] = mn;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(Ps + (tx * 4 + j) * QT + ty * 4) =
          make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) o[i][j] *= corr[i];
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < KT; ++j) {
      const float4 pv = *reinterpret_cast<const float4*>(Ps + j * QT + ty * 4);
      const float4 va = *reinterpret_cast<const float4*>(Vs + j * HD + tx * 8);
      const float4 vb2 = *reinterpret_cast<const float4*>(Vs + j * HD + tx * 8 + 4);
      const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
      const float vr[8] = {va.x, va.y, va.z, va.w, vb2.x, vb2.y, vb2.z, vb2.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int d = 0; d < 8; ++d) o[i][d] = fmaf(pa[i], vr[d], o[i][d]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t t = qt0 + ty * 4 + i;
    if (t >= a.n) continue;
    float* op = a.out + (t * a.n_heads + h) * HD + tx * 8;
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int d = 0; d < 8; ++d) op[d] = o[i][d] * inv;
  }
}

}  // namespace

cudaError_t qkv_rope_launch(const QkvArgs& a, cudaStream_t s) {
  if (a.hd > 256 || (a.hd & 31) || a.n <= 0) return cudaErrorInvalidValue;
  dim3 grid((unsigned)a.n, (unsigned)(a.n_heads + a.n_kv));
  qkv_rope_kernel<<<grid, a.hd, 0, s>>>(a);
  return cudaGetLastError();
}

size_t attn_decode_partial_floats(int n_kv, int n_heads, int hd, int max_splits) {
  return (size_t)n_kv * max_splits * (n_heads / n_kv) * 130 + (size_t)0 * hd;
}

cudaError_t attn_decode_launch(const AttnArgs& a, cudaStream_t s) {
  if (a.hd != 128 || a.n_heads % a.n_kv || a.n_heads / a.n_kv > kMaxGroup || a.max_splits < 1 ||
      a.max_splits > 32)
    return cudaErrorInvalidValue;
  if (a.q_norm && (!a.k_norm || !a.rope || !a.k_new || !a.v_new || !a.kc_w || !a.vc_w))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.n_kv, (unsigned)a.max_splits);
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel, a);
}

cudaError_t attn_prefill_launch(const AttnArgs& a, cudaStream_t s) {
  if (a.hd != HD || a.n_heads % a.n_kv || a.n <= 0) return cudaErrorInvalidValue;
  const size_t smem = (size_t)(HD * QT + HD * KT + KT * HD + KT * QT) * sizeof(float);
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = dev;
  }
  dim3 grid((unsigned)a.n_heads, (unsigned)((a.n + QT - 1) / QT));
  attn_prefill_kernel<<<grid, 256, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace rpgc
