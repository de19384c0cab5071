// k_attn.cu -- QK-norm + RoPE + KV-cache write, and GQA attention over the
// device KV cache (decode: split-K flash-decode; prefill: tiled causal).
//
// Reference: QK-norm before RoPE (src/qwen3.cc:141-152), half-split RoPE
// (src/kernels.h:108-120), cache layout ((l*nkv + h)*max_seq + pos)*hd
// (src/kv_cache.cc:29-33), AttentionFromCache with a softmax over [0, pos]
// (src/qwen3.cc:79-117).
#include <cooperative_groups.h>
#include <cstdlib>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "attn_dev.cuh"
#include "common.cuh"
#include "kernels.h"
#include "tc_dev.cuh"

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
  const int h = (int)blockIdx.y + (a.kv_only ? a.n_heads : 0), i = threadIdx.x, hd = a.hd, half = hd >> 1;
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

  // batched decode: session z = blockIdx.z (its rows of q / k_new / v_new /
  // out, its cache and state); otherwise z = 0 and the single-session fields
  const int64_t z = blockIdx.z;
  const AttnBatchEntry* be = a.batch ? a.batch + z : nullptr;
  const DecodeState* st = be ? be->state : a.state;
  const int64_t max_seq = be ? be->max_seq : a.max_seq;
  const int64_t loff = be ? (int64_t)a.layer * a.n_kv * max_seq * 128 : 0;
  const float* kcache = be ? be->kc + loff : a.kc;
  const float* vcache = be ? be->vc + loff : a.vc;
  float* kc_w = be ? be->kc + loff : a.kc_w;
  float* vc_w = be ? be->vc + loff : a.vc_w;
  const float* qz = a.q + z * a.n_heads * 128;
  const float* knz = a.k_new ? a.k_new + z * a.n_kv * 128 : nullptr;
  const float* vnz = a.v_new ? a.v_new + z * a.n_kv * 128 : nullptr;
  float* outz = a.out + z * a.n_heads * 128;
  int32_t* err = be ? be->err : a.err;  // a batched session's waits report to that session
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
  const float* kb = kcache + (int64_t)kh * max_seq * 128;
  const float* vb = vcache + (int64_t)kh * max_seq * 128;

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
  if (be && be->stall && a.layer == 0 && tid == 0) {
    // test hook: a bounded wait on a barrier that nothing completes gives up
    // and flags this session's error, which its caller reports
    __shared__ __align__(8) uint64_t never;
    mbar_init(&never, 1);
    fence_barrier_init();
    mbar_wait(&never, 0, err);
  }
  if (st && !st->active) {  // the whole cluster leaves together, copies drained
    if (tid == 0 && c0 < c1) mbar_wait(&bar, 0, err);
    return;
  }
  // query heads of this kv head (normalised and rotated when fused)
  for (int g = warp; g < G; g += kAWarps) {
    float4 v = *reinterpret_cast<const float4*>(qz + (kh * G + g) * 128 + 4 * lane);
    if (fused) v = norm_rope_head(v, a.q_norm, cs, a.eps, lane);
    *reinterpret_cast<float4*>(&qs[g][4 * lane]) = v;
  }
  float4 knew = make_float4(0.f, 0.f, 0.f, 0.f), vnew = knew;
  if (owner && warp == kAWarps - 1) {
    // the new token's k/v: normalise + rotate k, write both into the cache
    knew = *reinterpret_cast<const float4*>(knz + kh * 128 + 4 * lane);
    knew = norm_rope_head(knew, a.k_norm, cs, a.eps, lane);
    vnew = *reinterpret_cast<const float4*>(vnz + kh * 128 + 4 * lane);
    const int64_t off = ((int64_t)kh * max_seq + pos) * 128 + 4 * lane;
    *reinterpret_cast<float4*>(kc_w + off) = knew;
    *reinterpret_cast<float4*>(vc_w + off) = vnew;
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
    mbar_wait(&bar, phase, err);
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
      outz[(kh * G + g) * 128 + d] = O / Ls;
    }
  }
  cluster.sync();  // keep every CTA's shared memory alive until rank 0 is done
}

// --------------------------------------------------------------- prefill
// Causal attention of n new tokens over the cache (keys [0, pos0 + t]) on the
// tensor cores: warp-level mma.sync m16n8k16, fp16 operands, fp32
// accumulators.  Scores and the probability-weighted sum keep fp32-class
// accuracy by the three-product split used by the prefill matmul: every
// operand x = xh + xl (fp16 hi, fp16 residual), products Ah Bh + Ah Bl + Al Bh
// (the dropped Al Bl and the roundings leave ~2^-21 of sum |a b|).  The
// online softmax (running max, rescaled sums) is fp32 in registers, as in the
// reference's AttentionFromCache (src/qwen3.cc:79-117: scores q.k/sqrt(hd),
// softmax, sum of p v).
//
// grid (n_heads, ceil(n/64)), 128 threads: warp w owns queries 16w..16w+15 of
// the CTA's 64; per 64-key tile the CTA stages K and V as fp16 hi/lo rows
// [key][dim] (padded to 136 halves: conflict-free ldmatrix); each warp then
// forms S = Q K^T (16 x 64), the softmax update and O += P V (16 x 128), the
// P fragments taken straight from the S accumulators.  blockIdx.y = 0 takes
// the last (heaviest) query tile.  P enters the split scaled by 2^14 (p <= 1
// stays below the fp16 maximum, and p down to 2^-38 keeps a normal lo half);
// the final 1 / (2^14 l) removes it exactly.
constexpr int QT = 64, KT = 64, HD = 128, KP = HD + 8;
constexpr float kPScale = 16384.0f;

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// (a, b) -> fp16 pairs hi = fp16(a, b), lo = fp16(a - hi, b - hi).
__device__ __forceinline__ void split2(float a, float b, uint32_t* hi, uint32_t* lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 f = __half22float2(h);
  *hi = h2_bits(h);
  *lo = h2_bits(__floats2half2_rn(a - f.x, b - f.y));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Four 8x8 fp16 matrices (rows of 16 bytes at the lanes' addresses).
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__global__ void __launch_bounds__(128, 2) attn_prefill_kernel(const AttnArgs a) {
  grid_dep_wait();  // launched as a programmatic dependent: q and the cache come from earlier kernels
  extern __shared__ __align__(16) __half hsm[];
  __half* Kh = hsm;            // [KT][KP]
  __half* Kl = Kh + KT * KP;
  __half* Vh = Kl + KT * KP;
  __half* Vl = Vh + KT * KP;
  const int h = blockIdx.x;
  const int64_t qt0 = (int64_t)(gridDim.y - 1 - blockIdx.y) * QT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int G = a.n_heads / a.n_kv, kh = h / G;
  const float scale = 1.0f / sqrtf((float)HD);
  const int64_t qpos0 = a.pos0 + qt0;
  const int64_t nq = min((int64_t)QT, a.n - qt0);
  const int64_t key_end = qpos0 + nq;  // keys [0, key_end)
  const float* kb = a.kc + (int64_t)kh * a.max_seq * HD;
  const float* vb = a.vc + (int64_t)kh * a.max_seq * HD;

  // the warp's query rows r0 = 16 w + g and r1 = r0 + 8 as A fragments, k16
  // step kk: {(r0, 2t..), (r1, 2t..), (r0, 8+2t..), (r1, 8+2t..)} of dims 16kk..
  // With a.q_norm the rows arrive raw and get the QK-norm and RoPE here, with
  // qkv_rope_kernel's float operations: the four lanes of a quad hold a row's
  // 128 dims (sum of squares over the quad, in double), and dims i and i + 64
  // sit in steps kk and kk + 4 of the same lane.
  const int r0 = 16 * warp + g;
  uint32_t qh[8][4], ql[8][4];
  const float* qrow[2];
  float qsc[2] = {1.0f, 1.0f};
  const float* qcs[2] = {nullptr, nullptr};
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = r0 + 8 * hr;
    qrow[hr] = row < nq ? a.q + ((qt0 + row) * a.n_heads + h) * HD : nullptr;
    if (a.q_norm) {
      double ss = 0.0;
      if (qrow[hr])
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const float2 v = *reinterpret_cast<const float2*>(qrow[hr] + 16 * kk + 8 * hf + 2 * t);
            ss += (double)v.x * v.x + (double)v.y * v.y;
          }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      qsc[hr] = (float)(1.0 / sqrt(ss / (double)HD + (double)a.eps));
      qcs[hr] = a.rope + (row < nq ? qpos0 + row : qpos0) * HD;  // hd/2 cos then hd/2 sin
    }
  }
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int hr = e & 1, col = 16 * kk + 8 * (e >> 1) + 2 * t;
      float2 v = make_float2(0.f, 0.f);
      if (qrow[hr]) {
        v = *reinterpret_cast<const float2*>(qrow[hr] + col);
        if (a.q_norm) {
          const int pc = col ^ 64;  // the rotation partner dims
          const float2 pv = *reinterpret_cast<const float2*>(qrow[hr] + pc);
          const float2 gv = *reinterpret_cast<const float2*>(a.q_norm + col);
          const float2 gp = *reinterpret_cast<const float2*>(a.q_norm + pc);
          const float y0 = v.x * qsc[hr] * gv.x, y1 = v.y * qsc[hr] * gv.y;
          const float p0 = pv.x * qsc[hr] * gp.x, p1 = pv.y * qsc[hr] * gp.y;
          const int j = col & 63;
          const float c0 = qcs[hr][j], c1 = qcs[hr][j + 1], s0 = qcs[hr][64 + j], s1 = qcs[hr][64 + j + 1];
          if (col < 64) {
            v.x = __fsub_rn(__fmul_rn(y0, c0), __fmul_rn(p0, s0));
            v.y = __fsub_rn(__fmul_rn(y1, c1), __fmul_rn(p1, s1));
          } else {
            v.x = __fadd_rn(__fmul_rn(y0, c0), __fmul_rn(p0, s0));
            v.y = __fadd_rn(__fmul_rn(y1, c1), __fmul_rn(p1, s1));
          }
        }
      }
      split2(v.x, v.y, &qh[kk][e], &ql[kk][e]);
    }
  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
  float m0 = kNegBig, m1 = kNegBig, l0 = 0.0f, l1 = 0.0f;  // rows r0, r1 (l: this lane's columns)
  const int64_t qp0 = qpos0 + r0, qp1 = qp0 + 8;
  // ldmatrix row addresses: lane L gives row L & 7 of matrix L >> 3
  const int mi = lane >> 3, mr = lane & 7;
  const uint32_t kh_base = smem_u32(Kh), kl_base = smem_u32(Kl), vh_base = smem_u32(Vh), vl_base = smem_u32(Vl);
  // S operand: matrices (keys +0, dims +0), (keys +0, dims +8), (keys +8, dims +0), (keys +8, dims +8)
  const uint32_t koff = (uint32_t)(((8 * (mi >> 1) + mr) * KP + 8 * (mi & 1)) * 2);
  // PV operand (transposed): (keys +0, dims +0), (keys +8, dims +0), (keys +0, dims +8), (keys +8, dims +8)
  const uint32_t voff = (uint32_t)(((8 * (mi & 1) + mr) * KP + 8 * (mi >> 1)) * 2);

  for (int64_t k0 = 0; k0 < key_end; k0 += KT) {
    __syncthreads();  // the previous tile's fragments are all read
    for (int idx = tid; idx < KT * (HD / 4); idx += 128) {
      const int j = idx >> 5, c = idx & 31;  // key j, dims 4c .. 4c + 3
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (k0 + j < key_end) {
        kv = *reinterpret_cast<const float4*>(kb + (k0 + j) * HD + 4 * c);
        vv = *reinterpret_cast<const float4*>(vb + (k0 + j) * HD + 4 * c);
      }
      uint32_t h0, l0w, h1, l1w;
      split2(kv.x, kv.y, &h0, &l0w);
      split2(kv.z, kv.w, &h1, &l1w);
      *reinterpret_cast<uint2*>(Kh + j * KP + 4 * c) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(Kl + j * KP + 4 * c) = make_uint2(l0w, l1w);
      split2(vv.x, vv.y, &h0, &l0w);
      split2(vv.z, vv.w, &h1, &l1w);
      *reinterpret_cast<uint2*>(Vh + j * KP + 4 * c) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(Vl + j * KP + 4 * c) = make_uint2(l0w, l1w);
    }
    __syncthreads();
    // ---- S = Q K^T: n-tile n = keys 8n .. 8n + 7 of the tile
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const uint32_t off = koff + (uint32_t)((16 * np * KP + 16 * kk) * 2);
        uint32_t bh[4], bl[4];
        ldsm4(kh_base + off, bh);
        ldsm4(kl_base + off, bl);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float* c = sc[2 * np + q];
          mma16816(c, qh[kk], bh[2 * q], bh[2 * q + 1]);
          mma16816(c, qh[kk], bl[2 * q], bl[2 * q + 1]);
          mma16816(c, ql[kk], bh[2 * q], bh[2 * q + 1]);
        }
      }
    // ---- scale, causal mask, online softmax
    float mx0 = kNegBig, mx1 = kNegBig;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t key = k0 + 8 * n + 2 * t + (c & 1);
        const int64_t qp = c < 2 ? qp0 : qp1;
        const float v = (key <= qp && key < key_end) ? sc[n][c] * scale : kNegBig;
        sc[n][c] = v;
        if (c < 2) mx0 = fmaxf(mx0, v);
        else mx1 = fmaxf(mx1, v);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float corr0 = expf(m0 - mn0), corr1 = expf(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    l0 *= corr0;
    l1 *= corr1;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= corr0;
      o[d][1] *= corr0;
      o[d][2] *= corr1;
      o[d][3] *= corr1;
    }
    // ---- O += P V, k16 step i = keys 16i .. 16i + 15 = n-tiles 2i, 2i + 1
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float p[8];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        p[4 * q] = expf(sc[2 * i + q][0] - m0);
        p[4 * q + 1] = expf(sc[2 * i + q][1] - m0);
        p[4 * q + 2] = expf(sc[2 * i + q][2] - m1);
        p[4 * q + 3] = expf(sc[2 * i + q][3] - m1);
      }
      l0 += (p[0] + p[1]) + (p[4] + p[5]);
      l1 += (p[2] + p[3]) + (p[6] + p[7]);
      uint32_t ah[4], al[4];
      split2(p[0] * kPScale, p[1] * kPScale, &ah[0], &al[0]);  // (r0, keys 2t..)
      split2(p[2] * kPScale, p[3] * kPScale, &ah[1], &al[1]);  // (r1, keys 2t..)
      split2(p[4] * kPScale, p[5] * kPScale, &ah[2], &al[2]);  // (r0, keys 8+2t..)
      split2(p[6] * kPScale, p[7] * kPScale, &ah[3], &al[3]);  // (r1, keys 8+2t..)
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const uint32_t off = voff + (uint32_t)((16 * i * KP + 16 * dp) * 2);
        uint32_t bh[4], bl[4];
        ldsm4_t(vh_base + off, bh);
        ldsm4_t(vl_base + off, bl);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float* c = o[2 * dp + q];
          mma16816(c, ah, bh[2 * q], bh[2 * q + 1]);
          mma16816(c, ah, bl[2 * q], bl[2 * q + 1]);
          mma16816(c, al, bh[2 * q], bh[2 * q + 1]);
        }
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / (l0 * kPScale), inv1 = 1.0f / (l1 * kPScale);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = r0 + 8 * hr;
    if (row >= nq) continue;
    float* op = a.out + ((qt0 + row) * a.n_heads + h) * HD + 2 * t;
    const float inv = hr ? inv1 : inv0;
#pragma unroll
    for (int d = 0; d < 16; ++d)
      *reinterpret_cast<float2*>(op + 8 * d) = make_float2(o[d][2 * hr] * inv, o[d][2 * hr + 1] * inv);
  }
}

// --------------------------------------------------------------- prefill, tcgen05
// The same attention (same split, same 2^14 probability scale) on the
// 5th-generation tensor cores (tcgen05, TMEM accumulators).  One CTA of 8
// warps per (head, 128-query tile), heaviest tiles first.  All warps stage
// operands; query row t is TMEM lane t of the accumulators, and threads t and
// t + 128 share it (keys 0-31 and 32-63 of each tile, columns 0-63 and 64-127
// of the output).  Q gets its QK-norm and RoPE as it is staged and stays in
// shared memory as hi/lo halves; K, V^T and P are fp16 hi/lo K-major tiles
// with the 128-byte swizzle (V is transposed as it is staged, so that both
// products read K-major operands).  Per 64-key tile i, pipelined so that the
// tensor core works while the CUDA cores stage and run the softmax:
//   A. stage K(i + 1) and V(i) (two buffers of each);
//   B. one thread issues S(i + 1) = Q K(i + 1)^T (M = 128, N = 64; 8 k16
//      steps x 3 products) into the other of two TMEM S buffers;
//   C. wait for S(i) (issued one tile earlier);
//   D. a row's two threads read its S(i) row, mask it (keys past the row's
//      position or past the chunk), update the running max and sums and form
//      P = exp(s - max) 2^14 in registers -- while the tensor core runs
//      O += P(i - 1) V(i - 1) and S(i + 1);
//   E. wait for that product, write P(i) as an fp16 hi/lo row, rescale the
//      row of O (TMEM) by exp(old max - new max) unless no row of the warp
//      changed its max;
//   F. one thread issues O += P(i) V(i) (M = 128, N = 128; 4 k16 steps x 3
//      products).
// Each S buffer has its own mbarrier and each barrier completes once before
// it is waited on; all waits are bounded.
constexpr int TQ = 128;
constexpr int kQPanel = TQ * 128;     // one 64-dim panel of Q: 128 rows x 128 B
constexpr int kKPanel = KT * 128;     // one 64-dim panel of K: 64 rows x 128 B
constexpr int kKBuf = 4 * kKPanel;    // Kh and Kl, 2 panels each
constexpr int kVTile = HD * 128;      // V^T: 128 dim rows x 64 keys (128 B)
constexpr int kVBuf = 2 * kVTile;     // Vh and Vl
constexpr int kPTile = TQ * 128;      // P: 128 query rows x 64 keys
constexpr int kTcBytes = 4 * kQPanel + 2 * kKBuf + 2 * kVBuf + 2 * kPTile;
constexpr int kTcSmem = kTcBytes + 1024 + 64;  // + alignment slack, + barriers
constexpr uint32_t kTcCols = 256;  // S buffers at columns 0 and 192 (64 each), O at 64 (128)
// instruction descriptors: fp16 x fp16 -> fp32, both K-major, M = 128
constexpr uint32_t kIdS = (1u << 4) | ((uint32_t)(KT >> 3) << 17) | ((uint32_t)(TQ >> 4) << 24);
constexpr uint32_t kIdO = (1u << 4) | ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(TQ >> 4) << 24);
static_assert(kTcSmem + 2 * TQ * 4 <= 227 * 1024, "attention smem");

__global__ void __launch_bounds__(256, 1) attn_prefill_tc_kernel(const AttnArgs a) {
  grid_dep_wait();  // launched as a programmatic dependent: q and the cache come from earlier kernels
  using namespace tc;
  extern __shared__ uint8_t tsm_raw[];
  uint8_t* sb = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Qh = sb;                 // 2 panels
  uint8_t* Ql = Qh + 2 * kQPanel;
  uint8_t* Kb = Ql + 2 * kQPanel;   // [2] x (Kh 2 panels, Kl 2 panels)
  uint8_t* Vb = Kb + 2 * kKBuf;     // [2] x (Vh, Vl)
  uint8_t* Ph = Vb + 2 * kVBuf;
  uint8_t* Pl = Ph + kPTile;
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sb + kTcBytes);  // [2], one per S buffer
  uint64_t* bar_o = bar_s + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_s + 3);
  __shared__ float red[2][TQ];  // the two halves' maxima, at the end their sums

  const int h = blockIdx.x;
  const int64_t qt0 = (int64_t)(gridDim.y - 1 - blockIdx.y) * TQ;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.n_heads / a.n_kv, kh = h / G;
  const float scale = 1.0f / sqrtf((float)HD);
  const int64_t qpos0 = a.pos0 + qt0;
  const int64_t nq = min((int64_t)TQ, a.n - qt0);
  const int64_t key_end = qpos0 + nq;  // keys [0, key_end)
  const int T = (int)((key_end + KT - 1) / KT);  // key tiles
  const float* kbase = a.kc + (int64_t)kh * a.max_seq * HD;
  const float* vbase = a.vc + (int64_t)kh * a.max_seq * HD;

  if (tid == 0) {
    mbar_init(&bar_s[0], 1);
    mbar_init(&bar_s[1], 1);
    mbar_init(bar_o, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // ---- Q: warp w stages rows w + 8 u (u = 0..15) in two batches of 8, every
  // load of a batch (q, the position's cosines and sines) in flight before the
  // first norm; lane l holds dims 4l .. 4l + 3 (rows past the chunk are zeros)
  {
    const float4 gq = a.q_norm ? *reinterpret_cast<const float4*>(a.q_norm + 4 * lane) : make_float4(1.f, 1.f, 1.f, 1.f);
    const int ci = (4 * lane) & 63;
#pragma unroll 1
    for (int bt = 0; bt < 2; ++bt) {
      float4 qv[8], cv[8], sn[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int row = warp + 8 * (8 * bt + u);
        qv[u] = cv[u] = sn[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < nq) {
          qv[u] = *reinterpret_cast<const float4*>(a.q + ((qt0 + row) * a.n_heads + h) * HD + 4 * lane);
          if (a.q_norm) {
            const float* cs = a.rope + (qpos0 + row) * HD;
            cv[u] = *reinterpret_cast<const float4*>(cs + ci);
            sn[u] = *reinterpret_cast<const float4*>(cs + 64 + ci);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int row = warp + 8 * (8 * bt + u);
        float4 v = qv[u];
        if (row < nq && a.q_norm) v = norm_rope_head_pre(v, gq, cv[u], sn[u], a.eps, lane);  // warp-uniform
        uint32_t h0, l0, h1, l1;
        split2(v.x, v.y, &h0, &l0);
        split2(v.z, v.w, &h1, &l1);
        const int d = 4 * lane;
        const uint32_t off = (uint32_t)((d >> 6) * kQPanel) + swz(row, (d & 63) >> 3) + (uint32_t)((d & 7) * 2);
        *reinterpret_cast<uint2*>(Qh + off) = make_uint2(h0, h1);
        *reinterpret_cast<uint2*>(Ql + off) = make_uint2(l0, l1);
      }
    }
  }

  // K of tile kt into buffer kt & 1 (4 items of (key, 8 dims) per thread) and
  // V^T of tile vt into buffer vt & 1 (one 8-key x 4-dim block per thread:
  // warp = 8-key chunk, lane = 4 dims, transposed in registers); every load
  // in flight before the first conversion.  A tile index < 0 or >= T skips.
  auto stage = [&](int kt, int vt) {
    float4 kx[8], vx[8];
    const bool dok = kt >= 0 && kt < T, dov = vt >= 0 && vt < T;
    const int64_t k0 = (int64_t)kt * KT, v0 = (int64_t)vt * KT;
    if (dok) {
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int idx = it * 256 + tid, j = idx >> 4, c = idx & 15;
        const bool ok = k0 + j < key_end;
        const float4* kp = reinterpret_cast<const float4*>(kbase + (k0 + (ok ? j : 0)) * HD + 8 * c);
        kx[2 * it] = ok ? kp[0] : make_float4(0.f, 0.f, 0.f, 0.f);
        kx[2 * it + 1] = ok ? kp[1] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (dov) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t key = v0 + 8 * warp + i;
        vx[i] = key < key_end ? *reinterpret_cast<const float4*>(vbase + key * HD + 4 * lane)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (dok) {
      uint8_t* Kh = Kb + (kt & 1) * kKBuf;
      uint8_t* Kl = Kh + 2 * kKPanel;
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int idx = it * 256 + tid, j = idx >> 4, c = idx & 15;
        const float kv[8] = {kx[2 * it].x, kx[2 * it].y, kx[2 * it].z, kx[2 * it].w,
                             kx[2 * it + 1].x, kx[2 * it + 1].y, kx[2 * it + 1].z, kx[2 * it + 1].w};
        uint4 hi, lo;
        split8(kv, &hi, &lo);
        const uint32_t off = (uint32_t)((c >> 3) * kKPanel) + swz(j, c & 7);
        *reinterpret_cast<uint4*>(Kh + off) = hi;
        *reinterpret_cast<uint4*>(Kl + off) = lo;
      }
    }
    if (dov) {
      uint8_t* Vh = Vb + (vt & 1) * kVBuf;
      uint8_t* Vl = Vh + kVTile;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float vv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) vv[i] = e == 0 ? vx[i].x : e == 1 ? vx[i].y : e == 2 ? vx[i].z : vx[i].w;
        uint4 hi, lo;
        split8(vv, &hi, &lo);
        const int d = 4 * lane + e;
        *reinterpret_cast<uint4*>(Vh + swz(d, warp)) = hi;
        *reinterpret_cast<uint4*>(Vl + swz(d, warp)) = lo;
      }
    }
  };
  // S(t) = Q K(t)^T into S buffer t & 1 (one thread)
  auto issue_s = [&](uint32_t tmem, int t) {
    const uint8_t* Kh = Kb + (t & 1) * kKBuf;
    const uint8_t* Kl = Kh + 2 * kKPanel;
    const uint32_t d = tmem + (uint32_t)((t & 1) * 192);
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      const int pn = kk >> 2, ko = (kk & 3) * 32;
      const uint64_t qh = sdesc(Qh + pn * kQPanel + ko), ql = sdesc(Ql + pn * kQPanel + ko);
      const uint64_t bh = sdesc(Kh + pn * kKPanel + ko), bl = sdesc(Kl + pn * kKPanel + ko);
      mma_f16(d, qh, bh, kIdS, kk > 0 ? 1u : 0u);
      mma_f16(d, qh, bl, kIdS, 1u);
      mma_f16(d, ql, bh, kIdS, 1u);
    }
    mma_commit(&bar_s[t & 1]);
  };

  stage(0, -1);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // Q and K(0) visible to the MMAs
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's lane quarter
  const int r = (warp & 3) * 32 + lane, hf = warp >> 2;  // query row = TMEM lane; key / column half
  const int64_t qp = qpos0 + r;
  if (tid == 0) issue_s(tmem, 0);
  float m = kNegBig, l = 0.0f;

  for (int i = 0; i < T; ++i) {
    const int64_t k0 = (int64_t)i * KT;
    // ---- A, B. K(i + 1) and V(i); S(i + 1).  K buffer (i + 1) & 1 was read by
    // S(i - 1), waited for in the previous pass; V buffer i & 1 by PV(i - 2).
    stage(i + 1, i);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();  // also: every thread is done with S buffer (i + 1) & 1 and with red
    tc_fence_after();
    if (tid == 0 && i + 1 < T) issue_s(tmem, i + 1);
    // ---- C, D. S(i): scale, causal mask, online softmax into registers
    mbar_wait_sleep(&bar_s[i & 1], (uint32_t)(i >> 1) & 1u, a.err);
    tc_fence_after();
    float sv[32];
    tmem_ld32(tl + (uint32_t)((i & 1) * 192 + 32 * hf), sv);
    float mx = kNegBig;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int64_t key = k0 + 32 * hf + j;
      if (key <= qp && key < key_end) mx = fmaxf(mx, sv[j] * scale);
    }
    red[hf][r] = mx;
    __syncthreads();
    const float mn = fmaxf(m, fmaxf(red[0][r], red[1][r])), corr = expf(m - mn);
    m = mn;
    l *= corr;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int64_t key = k0 + 32 * hf + j;
      const float pv = (key <= qp && key < key_end) ? expf(sv[j] * scale - mn) : 0.0f;
      l += pv;
      sv[j] = pv * kPScale;
    }
    // ---- E. PV(i - 1) done: P(i) into shared memory, O's row rescaled
    if (i > 0) {
      mbar_wait_sleep(bar_o, (uint32_t)(i - 1) & 1u, a.err);
      tc_fence_after();
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 hi, lo;
      split8(sv + 8 * c, &hi, &lo);
      *reinterpret_cast<uint4*>(Ph + swz(r, 4 * hf + c)) = hi;
      *reinterpret_cast<uint4*>(Pl + swz(r, 4 * hf + c)) = lo;
    }
    if (i > 0 && __any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll 1
      for (int q = 0; q < 2; ++q) {
        float t[32];
        const uint32_t col = 64 + (uint32_t)(64 * hf + 32 * q);
        tmem_ld32(tl + col, t);
#pragma unroll
        for (int j = 0; j < 32; ++j) t[j] *= corr;
        tmem_st32(tl + col, t);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the MMAs
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- F. O += P(i) V(i)
    if (tid == 0) {
      const uint8_t* Vh = Vb + (i & 1) * kVBuf;
      const uint8_t* Vl = Vh + kVTile;
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk) {
        const int ko = kk * 32;
        const uint64_t pa = sdesc(Ph + ko), pl = sdesc(Pl + ko), vh = sdesc(Vh + ko), vl = sdesc(Vl + ko);
        mma_f16(tmem + 64, pa, vh, kIdO, (i > 0 || kk > 0) ? 1u : 0u);
        mma_f16(tmem + 64, pa, vl, kIdO, 1u);
        mma_f16(tmem + 64, pl, vh, kIdO, 1u);
      }
      mma_commit(bar_o);
    }
  }
  mbar_wait_sleep(bar_o, (uint32_t)(T - 1) & 1u, a.err);
  tc_fence_after();
  red[hf][r] = l;
  __syncthreads();
  const float inv = 1.0f / ((red[0][r] + red[1][r]) * kPScale);
  float4* op = r < nq ? reinterpret_cast<float4*>(a.out + ((qt0 + r) * a.n_heads + h) * HD + 64 * hf) : nullptr;
#pragma unroll 1
  for (int q = 0; q < 2; ++q) {
    float t[32];
    tmem_ld32(tl + 64 + (uint32_t)(64 * hf + 32 * q), t);  // warp-wide: every lane loads
    if (op)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        op[8 * q + j] = make_float4(t[4 * j] * inv, t[4 * j + 1] * inv, t[4 * j + 2] * inv, t[4 * j + 3] * inv);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  }
}

}  // namespace

cudaError_t qkv_rope_launch(const QkvArgs& a, cudaStream_t s) {
  if (a.hd > 256 || (a.hd & 31) || a.n <= 0) return cudaErrorInvalidValue;
  dim3 grid((unsigned)a.n, (unsigned)(a.kv_only ? a.n_kv : a.n_heads + a.n_kv));
  const cudaError_t e_ = launch_pdl(qkv_rope_kernel, grid, dim3((unsigned)a.hd), 0, s, a);  // waits first thing
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
  int S = cluster_size<G>();
  if (a.batch) {
    // a batch has parallelism across sessions: split a session's positions only
    // as far as needed for two CTAs per SM (fewer splits, fewer merges; 64
    // sessions of the 4B shape decode 1.6x faster unsplit than in 16 splits)
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int nsm = 148;
    if (dev >= 0 && dev < 64) {
      if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
      if (sms[dev] > 0) nsm = sms[dev];
    }
    int want = 1;
    while (want < S && (int64_t)a.n_kv * want * a.nbatch < 2 * nsm) want *= 2;
    S = want;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.n_kv, (unsigned)S, (unsigned)(a.batch ? a.nbatch : 1));
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
  if (!a.batch && ((reinterpret_cast<uintptr_t>(a.kc) | reinterpret_cast<uintptr_t>(a.vc)) & 15))
    return cudaErrorInvalidValue;
  if (a.batch && (a.nbatch < 1 || a.nbatch > 65535 || !a.q_norm)) return cudaErrorInvalidValue;
  if (a.q_norm && (!a.k_norm || !a.rope || !a.k_new || !a.v_new || (!a.batch && (!a.kc_w || !a.vc_w))))
    return cudaErrorInvalidValue;
  switch (G) {
    case 1: return launch_decode<1>(a, s);
    case 2: return launch_decode<2>(a, s);
    case 4: return launch_decode<4>(a, s);
    case 8: return launch_decode<8>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

namespace {

cudaError_t launch_prefill_mma(const AttnArgs& a, cudaStream_t s) {
  const size_t smem = (size_t)4 * KT * KP * sizeof(__half);
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  dim3 grid((unsigned)a.n_heads, (unsigned)((a.n + QT - 1) / QT));
  return launch_pdl(attn_prefill_kernel, grid, dim3(128), smem, s, a);
}

cudaError_t launch_prefill_tc(const AttnArgs& a, cudaStream_t s) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  dim3 grid((unsigned)a.n_heads, (unsigned)((a.n + TQ - 1) / TQ));
  return launch_pdl(attn_prefill_tc_kernel, grid, dim3(256), (size_t)kTcSmem, s, a);
}

}  // namespace

// RPGC_ATTN_TC=1 (read at every call) selects the tcgen05 kernel; the
// default is the mma.sync kernel, which is faster on the 512-token prefill.
cudaError_t attn_prefill_launch(const AttnArgs& a, cudaStream_t s) {
  if (a.hd != HD || a.n_kv <= 0 || a.n_heads % a.n_kv || a.n <= 0) return cudaErrorInvalidValue;
  const char* tc = getenv("RPGC_ATTN_TC");
  const cudaError_t e_ = (tc && tc[0] == '1') ? launch_prefill_tc(a, s) : launch_prefill_mma(a, s);
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

}  // namespace rpgc
