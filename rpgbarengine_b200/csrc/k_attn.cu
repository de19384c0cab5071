// k_attn.cu -- QK-norm + RoPE + KV-cache write, and GQA attention over the
// device KV cache (decode: split-K flash-decode; prefill: tiled causal).
//
// Reference: QK-norm before RoPE (src/qwen3.cc:141-152), half-split RoPE
// (src/kernels.h:108-120), cache layout ((l*nkv + h)*max_seq + pos)*hd
// (src/kv_cache.cc:29-33), AttentionFromCache with a softmax over [0, pos]
// (src/qwen3.cc:79-117).
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "attn_dev.cuh"
#include "common.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

namespace cg = cooperative_groups;
using namespace attn;

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
// One thread-block cluster per kv head, S = 8 or 16 CTAs (splits of the
// positions [0, pos]), 8 warps each; hd == 128 (4 dims per lane), group G =
// n_heads / n_kv in {1, 2, 4, 8}.  Each CTA streams its K and V rows into
// shared memory with two bulk copies per tile of up to 64 positions.  A warp
// step scores PB = 32 / G positions against the G query heads at once: the
// 32 partial dot products of a lane are folded across the warp by a
// transpose-reduction (31 shuffles leave lane l with score l), so no score
// needs its own warp-wide sum.  Warps keep an online softmax; the CTA merges
// its warps in shared memory and cluster rank 0 merges the S CTAs through
// distributed shared memory, in a fixed order (deterministic).
constexpr int kMaxGroup = 8;
constexpr int kAWarps = 8;
constexpr int kTileP = 64;  // positions per K/V tile

template <int G>
__global__ void __launch_bounds__(kAWarps * 32, 2) attn_decode_kernel(const AttnArgs a) {
  constexpr int PB = 32 / G;  // positions per warp step
  extern __shared__ __align__(128) float kv_tile[];  // K [kTileP][128], then V
  float* Ks = kv_tile;
  float* Vs = kv_tile + kTileP * 128;
  __shared__ __align__(16) float qs[G][128];
  __shared__ __align__(16) float wo[kAWarps][G][128];
  __shared__ float wm[kAWarps][G], wl[kAWarps][G];
  __shared__ __align__(16) float cpart[G][132];  // merged o[128], m, l of this CTA
  __shared__ __align__(8) uint64_t bar;

  const DecodeState* st = a.state;
  cg::cluster_group cluster = cg::this_cluster();
  const int S = (int)gridDim.y, split = (int)blockIdx.y, kh = (int)blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The position (decode state) was written before the previous kernel
  // started, and cache rows below it by earlier steps: every kernel of the
  // decode step signals its dependents only after its own grid-dependency
  // wait, so the kernel two launches back has completed.  The first K/V tile
  // is therefore copied before this kernel's wait.
  const int pos = st ? st->pos : (int)a.pos0;
  const int L = pos + 1;  // keys [0, pos]
  const int chunk = (L + S - 1) / S;
  const int c0 = min(L, split * chunk), c1 = min(L, c0 + chunk);
  const float scale = 1.0f / sqrtf(128.0f);
  const bool fused = a.q_norm != nullptr;
  const bool owner = fused && c0 <= pos && pos < c1;  // this split holds the new token
  const float* cs = fused ? a.rope + (int64_t)pos * 128 : nullptr;
  const float* kb = a.kc + (int64_t)kh * a.max_seq * 128;
  const float* vb = a.vc + (int64_t)kh * a.max_seq * 128;

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    if (c0 < c1) {  // first tile (the new token's row is replaced in shared memory)
      const uint32_t bytes = (uint32_t)min(kTileP, c1 - c0) * 512u;
      const uint64_t pol = policy_evict_first();
      mbar_arrive_expect_tx(&bar, 2 * bytes);
      bulk_g2s(Ks, kb + (int64_t)c0 * 128, bytes, &bar, pol);
      bulk_g2s(Vs, vb + (int64_t)c0 * 128, bytes, &bar, pol);
    }
  }
  grid_dep_wait();
  grid_dep_launch();
  if (st && !st->active) {  // the whole cluster leaves together, copies drained
    if (tid == 0 && c0 < c1) mbar_wait(&bar, 0, a.err);
    return;
  }
  // query heads of this kv head (normalised and rotated when fused)
  for (int g = warp; g < G; g += kAWarps) {
    float4 v = *reinterpret_cast<const float4*>(a.q + (kh * G + g) * 128 + 4 * lane);
    if (fused) v = norm_rope_head(v, a.q_norm, cs, a.eps, lane);
    *reinterpret_cast<float4*>(&qs[g][4 * lane]) = v;
  }
  float4 knew = make_float4(0.f, 0.f, 0.f, 0.f), vnew = knew;
  if (owner && warp == kAWarps - 1) {
    // the new token's k/v: normalise + rotate k, write both into the cache
    knew = *reinterpret_cast<const float4*>(a.k_new + kh * 128 + 4 * lane);
    knew = norm_rope_head(knew, a.k_norm, cs, a.eps, lane);
    vnew = *reinterpret_cast<const float4*>(a.v_new + kh * 128 + 4 * lane);
    const int64_t off = ((int64_t)kh * a.max_seq + pos) * 128 + 4 * lane;
    *reinterpret_cast<float4*>(a.kc_w + off) = knew;
    *reinterpret_cast<float4*>(a.vc_w + off) = vnew;
  }
  __syncthreads();

  float4 q[G], o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    q[g] = *reinterpret_cast<const float4*>(&qs[g][4 * lane]);
    o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mh = kNegBig, lh = 0.0f;  // running max / sum of this lane's head lane / PB
  const int gl = lane / PB, jl = lane % PB;
  uint32_t phase = 0;
  for (int t0 = c0; t0 < c1; t0 += kTileP) {
    const int tn = min(kTileP, c1 - t0);
    if (tid == 0 && t0 != c0) {
      const uint32_t bytes = (uint32_t)tn * 512u;
      const uint64_t pol = policy_evict_first();
      mbar_arrive_expect_tx(&bar, 2 * bytes);
      bulk_g2s(Ks, kb + (int64_t)t0 * 128, bytes, &bar, pol);
      bulk_g2s(Vs, vb + (int64_t)t0 * 128, bytes, &bar, pol);
    }
    mbar_wait(&bar, phase, a.err);
    phase ^= 1u;
    if (owner && warp == kAWarps - 1 && pos >= t0 && pos < t0 + tn) {
      reinterpret_cast<float4*>(Ks + (pos - t0) * 128)[lane] = knew;
      reinterpret_cast<float4*>(Vs + (pos - t0) * 128)[lane] = vnew;
    }
    __syncthreads();
    for (int pb = warp * PB; pb < tn; pb += kAWarps * PB) {
      float val[32];
#pragma unroll
      for (int j = 0; j < PB; ++j) {
        const float4 k = pb + j < tn ? reinterpret_cast<const float4*>(Ks + (pb + j) * 128)[lane]
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int g = 0; g < G; ++g) val[g * PB + j] = dot4(q[g], k);
      }
      const bool valid = pb + jl < tn;
      const float tr = transpose_reduce(val, lane);  // every lane takes part
      const float sc = valid ? tr * scale : kNegBig;
      float mx = sc;
#pragma unroll
      for (int n = PB / 2; n >= 1; n >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, n));
      const float mn = fmaxf(mh, mx);
      const float corr = expf(mh - mn);
      const float pe = valid ? expf(sc - mn) : 0.0f;
      float ps = pe;
#pragma unroll
      for (int n = PB / 2; n >= 1; n >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, n);
      lh = lh * corr + ps;
      mh = mn;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float cg_ = __shfl_sync(0xffffffffu, corr, g * PB);
        o[g].x *= cg_;
        o[g].y *= cg_;
        o[g].z *= cg_;
        o[g].w *= cg_;
      }
#pragma unroll
      for (int j = 0; j < PB; ++j) {
        if (pb + j >= tn) break;  // warp-uniform
        const float4 v = reinterpret_cast<const float4*>(Vs + (pb + j) * 128)[lane];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float p = __shfl_sync(0xffffffffu, pe, g * PB + j);
          o[g].x += p * v.x;
          o[g].y += p * v.y;
          o[g].z += p * v.z;
          o[g].w += p * v.w;
        }
      }
    }
    __syncthreads();  // the tile buffers may be refilled
  }
  // ---- merge the warps of this CTA
#pragma unroll
  for (int g = 0; g < G; ++g) *reinterpret_cast<float4*>(&wo[warp][g][4 * lane]) = o[g];
  if (jl == 0) {
    wm[warp][gl] = mh;
    wl[warp][gl] = lh;
  }
  __syncthreads();
  for (int idx = tid; idx < G * 128; idx += kAWarps * 32) {
    const int g = idx >> 7, d = idx & 127;
    float M = kNegBig;
    for (int w = 0; w < kAWarps; ++w) M = fmaxf(M, wm[w][g]);
    float O = 0.0f, Ls = 0.0f;
    for (int w = 0; w < kAWarps; ++w) {
      const float f = expf(wm[w][g] - M);
      O += wo[w][g][d] * f;
      Ls += wl[w][g] * f;
    }
    cpart[g][d] = O;
    if (d == 0) {
      cpart[g][128] = M;
      cpart[g][129] = Ls;
    }
  }
  // ---- merge the CTAs of the cluster on rank 0 (distributed shared memory)
  cluster.sync();
  if (cluster.block_rank() == 0) {
    for (int idx = tid; idx < G * 128; idx += kAWarps * 32) {
      const int g = idx >> 7, d = idx & 127;
      float M = kNegBig;
      for (int r = 0; r < S; ++r) M = fmaxf(M, cluster.map_shared_rank(&cpart[g][128], r)[0]);
      float O = 0.0f, Ls = 0.0f;
      for (int r = 0; r < S; ++r) {
        const float* rp = cluster.map_shared_rank(&cpart[g][0], r);
        const float f = expf(rp[128] - M);
        O += rp[d] * f;
        Ls += rp[129] * f;
      }
      a.out[(kh * G + g) * 128 + d] = O / Ls;
    }
  }
  cluster.sync();  // keep every CTA's shared memory alive until rank 0 is done
}

// --------------------------------------------------------------- prefill
// grid (n_heads, ceil(n/64)), 256 threads, two CTAs per SM; hd == 128.  The
// causal work of a query tile grows with its index, so blockIdx.y = 0 takes
// the last (heaviest) tile: the long CTAs start in the first wave.
constexpr int QT = 64, KT = 64, HD = 128;

__global__ void __launch_bounds__(256, 2) attn_prefill_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) float fsm[];
  float* Qs = fsm;             // [HD][QT]
  float* Ks = Qs + HD * QT;    // [HD][KT]
  float* Vs = Ks + HD * KT;    // [KT][HD]
  float* Ps = Ks;              // [KT][QT], over the key tile once the scores are taken
  const int h = blockIdx.x;
  const int64_t qt0 = (int64_t)(gridDim.y - 1 - blockIdx.y) * QT;
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
    __syncthreads();  // every thread's scores are taken: the key tile becomes P
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
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

namespace {

// Cluster size per device: 16 splits where a 16-CTA cluster of the kernel
// can be scheduled, else the portable 8.
template <int G>
int cluster_size() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 8;
  if (!cached[dev]) {
    const int smem = 2 * kTileP * 128 * (int)sizeof(float);
    cudaFuncSetAttribute(attn_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(attn_decode_kernel<G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
    int sz = 8;
    if (cudaFuncSetAttribute(attn_decode_kernel<G>, cudaFuncAttributeNonPortableClusterSizeAllowed,
                             1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 16);
      cfg.blockDim = dim3(kAWarps * 32);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 1;
      at[0].val.clusterDim.y = 16;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel<G>, &cfg) == cudaSuccess && n >= 1)
        sz = 16;
    }
    cudaGetLastError();  // a refused probe leaves no error behind
    cached[dev] = sz;
  }
  return cached[dev];
}

template <int G>
cudaError_t launch_decode(const AttnArgs& a, cudaStream_t s) {
  const int S = cluster_size<G>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.n_kv, (unsigned)S);
  cfg.blockDim = dim3(kAWarps * 32);
  cfg.dynamicSmemBytes = 2 * kTileP * 128 * sizeof(float);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)S;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 2 : 1;
  const cudaError_t e_ = cudaLaunchKernelEx(&cfg, attn_decode_kernel<G>, a);
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

}  // namespace

cudaError_t attn_decode_launch(const AttnArgs& a, cudaStream_t s) {
  const int G = a.n_kv > 0 ? a.n_heads / a.n_kv : 0;
  if (a.hd != 128 || a.n_kv <= 0 || a.n_heads % a.n_kv) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.kc) | reinterpret_cast<uintptr_t>(a.vc)) & 15)
    return cudaErrorInvalidValue;
  if (a.q_norm && (!a.k_norm || !a.rope || !a.k_new || !a.v_new || !a.kc_w || !a.vc_w))
    return cudaErrorInvalidValue;
  switch (G) {
    case 1: return launch_decode<1>(a, s);
    case 2: return launch_decode<2>(a, s);
    case 4: return launch_decode<4>(a, s);
    case 8: return launch_decode<8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t attn_prefill_launch(const AttnArgs& a, cudaStream_t s) {
  if (a.hd != HD || a.n_heads % a.n_kv || a.n <= 0) return cudaErrorInvalidValue;
  static_assert(KT * QT <= HD * KT, "P fits the key tile");
  const size_t smem = (size_t)(HD * QT + HD * KT + KT * HD) * sizeof(float);
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
  const cudaError_t e_ = cudaGetLastError();
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

}  // namespace rpgc
