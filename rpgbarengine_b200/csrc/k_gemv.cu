// k_gemv.cu -- decode GEMV over raw ggml blocks (batch 1), sm_100a.
//
// Replaces the reference's fused dequant dot-row (src/matmul_avx2.cc:95-289,
// dispatched per row by QuantMatrix::MatVec/MatMulBatch, src/model.cc:23-69).
//
// Data path.  Weights stay in their ggml block layout in HBM.  One CTA per SM
// (<= 112 KB of shared memory, so the next kernel's CTA fits beside it).  A
// producer warp streams row segments into a 4-stage shared-memory ring with
// bulk async copies (cp.async.bulk + mbarrier, evict-first L2 policy).  It
// does not wait for the previous kernel: weights do not depend on it, and with
// programmatic dependent launch the copies overlap the previous kernel's
// tail.  Consumer warps own one weight row per lane and split each row's
// blocks between warps, so activation reads are warp-uniform broadcasts.
// Weight reads are bank-conflict free: Q4_K slots are 16-byte aligned with an
// odd 16-byte pitch (128-bit loads); Q6_K rows whose length is 4 or 12 mod 16
// are assigned to lanes so that the 32 lanes of a warp start in 32 distinct
// banks (32-bit loads).
//
// Work items are (32-row tile, K range) pairs.  Matrices with few tiles are
// split along K across CTAs; the CTA that completes a tile last (atomic
// counter) adds the partial sums in a fixed order, so results are
// deterministic.
//
// Arithmetic.  The fp32 activation is turned, once per CTA, into a 24-bit
// fixed-point copy per group of 32 elements (power-of-two scale 2^(e-23),
// |A| < 2^23) held as three byte limbs A = 65536*A2 + 256*A1 + A0.  A block
// dot product is then 3 dp4a per 4 weights with exact int32 partial sums, and
// the ggml scales are applied per sub-block in fp32:
//   Q4_K  sum = s_g * (d*sc * S - dmin*m * sum(A))
//   Q6_K  sum = s_g * (d*sc) * (S - 32 * sum(A))       (q stored as 0..63)
//   Q8_0  sum = s_g * d * S
// The fixed-point rounding is 2^-24 of the group maximum, far inside the
// per-row gate max|d| / sum|a*w| <= 1e-5.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

constexpr int kNW = 8;             // consumer warps
constexpr int kThreads = (kNW + 1) * 32;
constexpr int kRPT = 32;           // rows per tile (one per lane)
constexpr int kMaxStages = 4;
constexpr int kSmemLimit = 112 * 1024;  // leaves room for the next kernel's CTA
constexpr int kStageMax = 20 * 1024;
constexpr int kMaxKParts = 8;

struct ActView {
  const uint32_t* l2;  // signed high limb words (4 elements each)
  const uint32_t* l1;
  const uint32_t* l0;
  const float* gs;     // per 32-group scale 2^(e-23)
  const int* sa32;     // per 32-group sum of A
  const int* sa16;     // per 16-group sum of A
  const float* xf;     // fp32 copy (F32 weights only)
};

struct SegInfo {
  int64_t item_begin;  // first global work item of this segment
  int64_t tile_begin;  // first global tile (counter index)
  int32_t tiles;       // 0 for the up half of a SwiGLU pair
  int32_t ks;          // K parts per tile
  int32_t be, bb;      // block elements / bytes
  int32_t nb;          // blocks per row
  int32_t cb;          // blocks per chunk
  int32_t nch;         // chunks per row
  int32_t slot;        // bytes per row slot in a stage
  int32_t perm;        // 1: permuted lane->row map (rows 4 or 12 mod 16 bytes)
};

struct Plan {
  SegInfo si[4];
  int64_t n_items;
  int32_t need_f32;
  int32_t split;       // some segment is split along K
  int32_t stages;      // ring depth (<= kMaxStages)
};

__device__ __forceinline__ float comb(int s2, int s1, int s0) {
  return (float)s2 * 65536.0f + (float)s1 * 256.0f + (float)s0;
}

// ---- per-unit dot products (one unit = one lane's row piece) -------------

// Byte k (0..11) of the Q4_K scale field held in three registers.
__device__ __forceinline__ uint32_t sbyte(uint32_t w0, uint32_t w1, uint32_t w2, int k) {
  const uint32_t w = k < 4 ? w0 : (k < 8 ? w1 : w2);
  return (w >> (8 * (k & 3))) & 0xFFu;
}
// get_scale_min_k4 on register-held scale bytes.
__device__ __forceinline__ void scale_min_regs(int j, uint32_t w0, uint32_t w1, uint32_t w2,
                                               uint32_t* sc, uint32_t* m) {
  if (j < 4) {
    *sc = sbyte(w0, w1, w2, j) & 63u;
    *m = sbyte(w0, w1, w2, j + 4) & 63u;
  } else {
    *sc = (sbyte(w0, w1, w2, j + 4) & 0x0Fu) | ((sbyte(w0, w1, w2, j - 4) >> 6) << 4);
    *m = (sbyte(w0, w1, w2, j + 4) >> 4) | ((sbyte(w0, w1, w2, j) >> 6) << 4);
  }
}

// Q4_K: unit = 64-element group g of a 256-element block (144 B, 16-aligned).
__device__ __forceinline__ float unit_q4k(const uint8_t* blk, int g, int e0, const ActView& a) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
  const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
  const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
  const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  uint32_t sc0, m0, sc1, m1;  // the 12 scale bytes are hdr.y, hdr.z, hdr.w
  scale_min_regs(2 * g, hdr.y, hdr.z, hdr.w, &sc0, &m0);
  scale_min_regs(2 * g + 1, hdr.y, hdr.z, hdr.w, &sc1, &m1);
  const int wb = e0 >> 2;
  const uint4* L2 = reinterpret_cast<const uint4*>(a.l2 + wb);
  const uint4* L1 = reinterpret_cast<const uint4*>(a.l1 + wb);
  const uint4* L0 = reinterpret_cast<const uint4*>(a.l0 + wb);
  int lo2 = 0, lo1 = 0, lo0 = 0, hi2 = 0, hi1 = 0, hi0 = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 x2 = L2[h], x1 = L1[h], x0 = L0[h];
    const uint4 y2 = L2[2 + h], y1 = L1[2 + h], y0 = L0[2 + h];
    const uint32_t a2[4] = {x2.x, x2.y, x2.z, x2.w}, a1[4] = {x1.x, x1.y, x1.z, x1.w},
                   a0[4] = {x0.x, x0.y, x0.z, x0.w};
    const uint32_t b2[4] = {y2.x, y2.y, y2.z, y2.w}, b1[4] = {y1.x, y1.y, y1.z, y1.w},
                   b0[4] = {y0.x, y0.y, y0.z, y0.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w = qw[4 * h + j];
      const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
      lo2 = dp4a_us(lo, a2[j], lo2);
      lo1 = dp4a_uu(lo, a1[j], lo1);
      lo0 = dp4a_uu(lo, a0[j], lo0);
      hi2 = dp4a_us(hi, b2[j], hi2);
      hi1 = dp4a_uu(hi, b1[j], hi1);
      hi0 = dp4a_uu(hi, b0[j], hi0);
    }
  }
  const float d = f16_bits_to_f32(hdr.x & 0xFFFFu), dmin = f16_bits_to_f32(hdr.x >> 16);
  const int grp = e0 >> 5;
  const float t0 = (d * (float)sc0) * comb(lo2, lo1, lo0) - (dmin * (float)m0) * (float)a.sa32[grp];
  const float t1 =
      (d * (float)sc1) * comb(hi2, hi1, hi0) - (dmin * (float)m1) * (float)a.sa32[grp + 1];
  return a.gs[grp] * t0 + a.gs[grp + 1] * t1;
}

// Q6_K: unit = one quarter of a 256-element block: half h, l-range
// [16*jb, 16*jb + 16), all four 32-element quadrants -> 64 elements in four
// 16-element sub-blocks (210-byte blocks, 2-byte aligned).
__device__ __forceinline__ float unit_q6k(const uint8_t* blk, int u, int e0, const ActView& a) {
  const int h = u >> 1, jb = u & 1;
  uint32_t qa[4], qb[4], qh[4], scw[2];
  lds_words<4>(blk + 64 * h + 16 * jb, qa);       // ql[l]      (quadrants 0, 2)
  lds_words<4>(blk + 64 * h + 32 + 16 * jb, qb);  // ql[l + 32] (quadrants 1, 3)
  lds_words<4>(blk + 128 + 32 * h + 16 * jb, qh);
  lds_words<2>(blk + 192 + 8 * h, scw);
  const float d = f16_bits_to_f32(lds_u32(blk + 208) & 0xFFFFu);
  const int wb = e0 >> 2;  // word of element 128*h of this block
  float acc = 0.0f;
#pragma unroll
  for (int qd = 0; qd < 4; ++qd) {
    const int aw = wb + 8 * qd + 4 * jb;
    const uint4 A2 = *reinterpret_cast<const uint4*>(a.l2 + aw);
    const uint4 A1 = *reinterpret_cast<const uint4*>(a.l1 + aw);
    const uint4 A0 = *reinterpret_cast<const uint4*>(a.l0 + aw);
    const uint32_t a2[4] = {A2.x, A2.y, A2.z, A2.w}, a1[4] = {A1.x, A1.y, A1.z, A1.w},
                   a0[4] = {A0.x, A0.y, A0.z, A0.w};
    int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const uint32_t A = qa[jj], B = qb[jj], H = qh[jj];
      uint32_t q;
      if (qd == 0) q = (A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
      else if (qd == 1) q = (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
      else if (qd == 2) q = ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
      else q = ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
      s2 = dp4a_us(q, a2[jj], s2);
      s1 = dp4a_uu(q, a1[jj], s1);
      s0 = dp4a_uu(q, a0[jj], s0);
    }
    const int sbi = jb + 2 * qd;  // scale index inside this half
    const int sc = (int)(int8_t)((scw[sbi >> 2] >> (8 * (sbi & 3))) & 0xFFu);
    const int e = e0 + 32 * qd + 16 * jb;
    acc += a.gs[e >> 5] * (d * (float)sc) * (comb(s2, s1, s0) - 32.0f * (float)a.sa16[e >> 4]);
  }
  return acc;
}

// Q8_0: unit = one 32-element block (34 B, 2-byte aligned).
__device__ __forceinline__ float unit_q8_0(const uint8_t* blk, int e0, const ActView& a) {
  uint32_t w[9];
  lds_words<9>(blk, w);
  const float d = f16_bits_to_f32(w[0] & 0xFFFFu);
  const int wb = e0 >> 2;
  int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t q = __funnelshift_r(w[j], w[j + 1], 16);
    s2 = dp4a_ss(q, a.l2[wb + j], s2);
    s1 = dp4a_su(q, a.l1[wb + j], s1);
    s0 = dp4a_su(q, a.l0[wb + j], s0);
  }
  return a.gs[e0 >> 5] * d * comb(s2, s1, s0);
}

// F32: unit = 32 elements, plain fp32 dot.
__device__ __forceinline__ float unit_f32(const uint8_t* p, int e0, const ActView& a) {
  const float4* w = reinterpret_cast<const float4*>(p);
  const float4* x = reinterpret_cast<const float4*>(a.xf + e0);
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 u = w[j], v = x[j];
    s += u.x * v.x + u.y * v.y + u.z * v.z + u.w * v.w;
  }
  return s;
}

__device__ __forceinline__ int units_per_block(uint32_t type) {
  return (type == kQ4_K || type == kQ6_K) ? 4 : 1;
}

// Row of lane `lane` in a tile: identity, or the permutation that puts the 32
// lanes of a warp in 32 distinct banks when rows are 4 or 12 mod 16 bytes
// (lanes l, l+8, l+16, l+24 then hold rows whose data start at different
// 4-byte offsets inside their 16-byte-aligned slots).
__device__ __forceinline__ int lane_row(int lane, int perm) {
  return perm ? 4 * (lane & 7) + (lane >> 3) : lane;
}

struct Item {
  int seg;        // segment (the gate for a SwiGLU pair)
  int64_t tile;   // tile index inside the segment
  int kp;         // K part
};

__device__ __forceinline__ Item locate(const GemvArgs& A, const Plan& P, int64_t t) {
  int k = 0;  // last segment owning items that starts at or before t
  for (int i = 1; i < A.nseg; ++i)
    if (P.si[i].tiles > 0 && t >= P.si[i].item_begin) k = i;
  const int64_t r = t - P.si[k].item_begin;
  Item it;
  it.seg = k;
  it.tile = r / P.si[k].ks;
  it.kp = (int)(r - it.tile * P.si[k].ks);
  return it;
}

// Chunk range [c0, c1) of K part kp.
__device__ __forceinline__ void kpart_chunks(const SegInfo& I, int kp, int* c0, int* c1) {
  const int per = (I.nch + I.ks - 1) / I.ks;
  *c0 = min(I.nch, kp * per);
  *c1 = min(I.nch, *c0 + per);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const GemvArgs A, const Plan P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = A.K;
  const bool need_f32 = P.need_f32 != 0;
  // ---- shared-memory carve-up (must match gemv_smem_bytes)
  uint8_t* p = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(p);
  uint64_t* empty = full + kMaxStages;
  const int kStages = P.stages;
  p += 128;
  float* red = reinterpret_cast<float*>(p);  // [2][kNW][32]
  p += 2 * kNW * 32 * 4;
  float* pair_buf = reinterpret_cast<float*>(p);  // [32] gate of a SwiGLU pair
  p += 32 * 4;
  double* dred = reinterpret_cast<double*>(p);  // [kNW]
  p += 16 * 8;
  int* flag = reinterpret_cast<int*>(p);
  p += 128;
  uint32_t* l2 = reinterpret_cast<uint32_t*>(p);
  p += K;
  uint32_t* l1 = reinterpret_cast<uint32_t*>(p);
  p += K;
  uint32_t* l0 = reinterpret_cast<uint32_t*>(p);
  p += K;
  float* gs = reinterpret_cast<float*>(p);
  p += (K / 32) * 4;
  int* sa32 = reinterpret_cast<int*>(p);
  p += (K / 32) * 4;
  int* sa16 = reinterpret_cast<int*>(p);
  p += (K / 16) * 4;
  float* xf = reinterpret_cast<float*>(p);
  if (need_f32) p += (size_t)K * 4;
  p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 127) & ~uintptr_t(127));
  uint8_t* stage_base = p;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kNW);
    }
    fence_barrier_init();
    grid_dep_launch();  // the next kernel may start its own weight prefetch
  }
  __syncthreads();

  if (warp == kNW) {
    // ============================== producer warp
    const uint64_t pol = policy_evict_first();
    uint32_t it = 0;
    for (int64_t t = blockIdx.x; t < P.n_items; t += gridDim.x) {
      const Item I0 = locate(A, P, t);
      const int passes = (A.seg[I0.seg].mode == kSwiGLU) ? 2 : 1;
      const SegInfo& I = P.si[I0.seg];  // chunking is identical within a pair
      const int64_t row0 = I0.tile * kRPT;
      const int r = lane_row(lane, I.perm);
      int c0, c1;
      kpart_chunks(I, I0.kp, &c0, &c1);
      for (int ps = 0; ps < passes; ++ps) {
        const GemvSeg& G = A.seg[I0.seg + ps];
        for (int c = c0; c < c1; ++c, ++it) {
          const int st = it % kStages;
          const uint32_t ph = (it / kStages) & 1u;
          if (it >= kStages) mbar_wait(&empty[st], ph ^ 1u, A.err);
          const int b0 = c * I.cb;
          const int nbk = min(I.cb, I.nb - b0);
          uint32_t bytes = 0;
          const uint8_t* src = nullptr;
          uint8_t* dst = nullptr;
          if (row0 + r < G.rows) {
            const uintptr_t s0 = reinterpret_cast<uintptr_t>(G.w) +
                                 (uintptr_t)(row0 + r) * G.row_bytes + (uintptr_t)b0 * I.bb;
            const uintptr_t a0 = s0 & ~uintptr_t(15);
            const uintptr_t a1 = (s0 + (uintptr_t)nbk * I.bb + 15) & ~uintptr_t(15);
            bytes = (uint32_t)(a1 - a0);
            src = reinterpret_cast<const uint8_t*>(a0);
            dst = stage_base + (size_t)st * kStageMax + (size_t)lane * I.slot;
          }
          const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
          if (lane == 0) mbar_arrive_expect_tx(&full[st], total);
          __syncwarp();
          if (bytes) bulk_g2s(dst, src, bytes, &full[st], pol);
        }
      }
    }
    return;
  }

  // ================================ consumer warps
  grid_dep_wait();
  const bool active = !A.active || *A.active != 0;
  const int ctid = threadIdx.x;  // 0 .. kNW*32-1
  float nscale = 1.0f;
  if (active) {
    // ---- optional RMSNorm scale of x (sum of squares in double)
    if (A.norm_w) {
      double ss = 0.0;
      for (int i = ctid; i < K; i += kNW * 32) {
        const float v = A.x[i];
        ss += (double)v * v;
      }
      ss = warp_sum(ss);
      if (lane == 0) dred[warp] = ss;
      asm volatile("bar.sync 1, %0;" ::"r"(kNW * 32));
      double tot = 0.0;
      for (int w = 0; w < kNW; ++w) tot += dred[w];
      nscale = (float)(1.0 / sqrt(tot / (double)K + (double)A.eps));
    }
    // ---- fixed-point activation limbs, one warp per 32-element group
    for (int g = warp; g < K / 32; g += kNW) {
      float h = A.x[g * 32 + lane];
      if (A.norm_w) h = h * nscale * A.norm_w[g * 32 + lane];
      if (need_f32) xf[g * 32 + lane] = h;
      const float amax = warp_max(fabsf(h));
      const uint32_t eb = (__float_as_uint(amax) >> 23) & 0xFFu;  // biased exponent
      int q = 0;
      float scale = 0.0f;
      if (eb >= 30 && eb < 255) {  // amax >= 2^-97 (tinier groups contribute nothing)
        // amax < 2^(eb-126): scaling by 2^(149-eb) keeps |q| < 2^23
        q = __float2int_rn(h * __uint_as_float((uint32_t)(276 - eb) << 23));
        q = max(-8388607, min(8388607, q));
        scale = __uint_as_float((eb - 22) << 23);  // 2^(eb-149)
      }
      const int sh = 8 * (lane & 3);
      uint32_t w0 = ((uint32_t)q & 0xFFu) << sh;
      uint32_t w1 = (((uint32_t)q >> 8) & 0xFFu) << sh;
      uint32_t w2 = (((uint32_t)(q >> 16)) & 0xFFu) << sh;
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        w0 |= __shfl_xor_sync(0xffffffffu, w0, o);
        w1 |= __shfl_xor_sync(0xffffffffu, w1, o);
        w2 |= __shfl_xor_sync(0xffffffffu, w2, o);
      }
      if ((lane & 3) == 0) {
        l0[g * 8 + (lane >> 2)] = w0;
        l1[g * 8 + (lane >> 2)] = w1;
        l2[g * 8 + (lane >> 2)] = w2;
      }
      int s16 = q;
#pragma unroll
      for (int o = 1; o <= 8; o <<= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
      const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
      if (lane == 0) {
        gs[g] = scale;
        sa32[g] = s32;
        sa16[2 * g] = s16;
      } else if (lane == 16) {
        sa16[2 * g + 1] = s16;
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kNW * 32));

  const ActView av{l2, l1, l0, gs, sa32, sa16, xf};
  uint32_t it = 0;
  int rb = 0;
  for (int64_t t = blockIdx.x; t < P.n_items; t += gridDim.x) {
    const Item I0 = locate(A, P, t);
    const SegInfo& I = P.si[I0.seg];
    const int passes = (A.seg[I0.seg].mode == kSwiGLU) ? 2 : 1;
    const int64_t row0 = I0.tile * kRPT;
    const int r = lane_row(lane, I.perm);
    int c0, c1;
    kpart_chunks(I, I0.kp, &c0, &c1);
    for (int ps = 0; ps < passes; ++ps) {
      const GemvSeg& G = A.seg[I0.seg + ps];
      const bool have = active && (row0 + r < G.rows);
      const int upb = units_per_block(G.type);
      float acc = 0.0f;
      for (int c = c0; c < c1; ++c, ++it) {
        const int st = it % kStages;
        const uint32_t ph = (it / kStages) & 1u;
        mbar_wait(&full[st], ph, A.err);
        const int b0 = c * I.cb;
        const int nbk = min(I.cb, I.nb - b0);
        if (have) {
          const uintptr_t s0 = reinterpret_cast<uintptr_t>(G.w) +
                               (uintptr_t)(row0 + r) * G.row_bytes + (uintptr_t)b0 * I.bb;
          const uint8_t* rowp =
              stage_base + (size_t)st * kStageMax + (size_t)lane * I.slot + (s0 & 15);
          const int nu = nbk * upb;
          for (int u = warp; u < nu; u += kNW) {
            const int bi = u / upb, sub = u - bi * upb;
            const uint8_t* blk = rowp + (size_t)bi * I.bb;
            const int eb = (b0 + bi) * I.be;  // element index of the block
            if (G.type == kQ4_K) acc += unit_q4k(blk, sub, eb + 64 * sub, av);
            else if (G.type == kQ6_K) acc += unit_q6k(blk, sub, eb + 128 * (sub >> 1), av);
            else if (G.type == kQ8_0) acc += unit_q8_0(blk, eb, av);
            else acc += unit_f32(blk, eb, av);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
      if (!active) continue;
      // ---- cross-warp reduction in fixed order
      float* rbuf = red + rb * kNW * 32;
      rbuf[warp * 32 + lane] = acc;
      asm volatile("bar.sync 1, %0;" ::"r"(kNW * 32));
      rb ^= 1;
      if (warp != 0) continue;
      float y = 0.0f;
#pragma unroll
      for (int w = 0; w < kNW; ++w) y += rbuf[w * 32 + lane];
      const int64_t row = row0 + r;
      if (I.ks == 1) {  // whole K in this CTA: epilogue now
        if (row < G.rows) {
          if (G.mode == kSwiGLU) pair_buf[lane] = y;
          else if (ps == 1) G.out[row] = silu_mul(pair_buf[lane], y);
          else if (G.mode == kAdd) G.out[row] += y;
          else G.out[row] = y;
        }
      } else {  // partial: park it; the CTA finishing the tile last combines
        A.partial[((I.item_begin + I0.tile * I.ks + I0.kp) * 2 + ps) * kRPT + lane] = y;
      }
    }
    if (!active || I.ks == 1 || warp != 0) continue;
    // ---- split tile: the CTA that completes it last sums the parts in order
    __threadfence();
    __syncwarp();
    if (lane == 0) {
      int* cnt = A.counters + (I.tile_begin + I0.tile);
      const int last = (atomicAdd(cnt, 1) == I.ks - 1);
      if (last) *cnt = 0;  // ready for the next launch
      flag[0] = last;
    }
    __syncwarp();
    if (flag[0]) {
      __threadfence();
      float y[2] = {0.0f, 0.0f};
      const float* base = A.partial + (I.item_begin + I0.tile * I.ks) * 2 * kRPT;
      for (int ps = 0; ps < passes; ++ps)
        for (int kp = 0; kp < I.ks; ++kp) y[ps] += __ldcg(base + (kp * 2 + ps) * kRPT + lane);
      const int64_t row = row0 + r;
      const GemvSeg& G = A.seg[I0.seg];
      if (row < G.rows) {
        if (passes == 2) A.seg[I0.seg + 1].out[row] = silu_mul(y[0], y[1]);
        else if (G.mode == kAdd) G.out[row] += y[0];
        else G.out[row] = y[0];
      }
    }
    __syncwarp();
  }
}

// Work decomposition shared by the launcher and the kernel.
bool make_plan(const GemvArgs& a, Plan* P, int sms) {
  int64_t tiles_total = 0;
  for (int i = 0; i < a.nseg; ++i) {
    const GemvSeg& G = a.seg[i];
    SegInfo& I = P->si[i];
    switch (G.type) {
      case kQ4_K: I.be = 256; I.bb = 144; break;
      case kQ6_K: I.be = 256; I.bb = 210; break;
      case kQ8_0: I.be = 32; I.bb = 34; break;
      case kF32: I.be = 32; I.bb = 128; break;
      default: return false;
    }
    if (a.K % I.be != 0 || a.K % 32 != 0) return false;
    I.nb = a.K / I.be;
    if ((int64_t)I.nb * I.bb != G.row_bytes) return false;
    const int max_cb = (kStageMax / kRPT - 64) / I.bb;
    if (max_cb < 1) return false;
    I.nch = (I.nb + max_cb - 1) / max_cb;
    I.cb = (I.nb + I.nch - 1) / I.nch;
    int slot = ((I.cb * I.bb + 32) + 15) & ~15;
    if (((slot >> 4) & 1) == 0) slot += 16;  // odd 16-byte pitch: conflict-free 128-bit loads
    if (slot * kRPT > kStageMax) return false;
    I.slot = slot;
    const int rm = (int)(G.row_bytes & 15);
    I.perm = (G.type == kQ6_K && (rm == 4 || rm == 12)) ? 1 : 0;
    const bool up_of_pair = (i > 0 && a.seg[i - 1].mode == kSwiGLU);
    if (up_of_pair) {
      if (G.rows != a.seg[i - 1].rows || G.type != a.seg[i - 1].type) return false;
      I.tiles = 0;
    } else {
      I.tiles = (int32_t)((G.rows + kRPT - 1) / kRPT);
      tiles_total += I.tiles;
    }
  }
  if (a.nseg > 0 && a.seg[a.nseg - 1].mode == kSwiGLU) return false;
  // split along K until there are about two work items per SM
  int ks = 1;
  while (tiles_total * ks < 2 * (int64_t)sms && ks < kMaxKParts) ks *= 2;
  int64_t items = 0, tiles = 0;
  P->split = 0;
  for (int i = 0; i < a.nseg; ++i) {
    SegInfo& I = P->si[i];
    if (I.tiles == 0) {  // up half of a pair mirrors the gate
      I.ks = P->si[i - 1].ks;
      I.item_begin = P->si[i - 1].item_begin;
      I.tile_begin = P->si[i - 1].tile_begin;
      continue;
    }
    I.ks = ks < I.nch ? ks : I.nch;
    if (a.partial == nullptr || a.counters == nullptr) I.ks = 1;
    if (I.ks > 1) P->split = 1;
    I.item_begin = items;
    I.tile_begin = tiles;
    items += (int64_t)I.tiles * I.ks;
    tiles += I.tiles;
  }
  P->n_items = items;
  if (P->split) {
    if ((size_t)items * 2 * kRPT > a.partial_floats || tiles > a.n_counters) return false;
  }
  P->need_f32 = 0;
  for (int i = 0; i < a.nseg; ++i) {
    if (a.seg[i].type == kF32) P->need_f32 = 1;
    if (reinterpret_cast<uintptr_t>(a.seg[i].w) & 15) return false;  // bulk copies need 16 B
  }
  return true;
}

int sm_count() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    sms[dev] = n > 0 ? n : 148;
  }
  return sms[dev];
}

}  // namespace

size_t gemv_act_bytes(int K, bool need_f32) {
  size_t b = 128 + 2 * kNW * 32 * 4 + 32 * 4 + 16 * 8 + 128;
  b += 3 * (size_t)K + (K / 32) * 8 + (K / 16) * 4;
  if (need_f32) b += (size_t)K * 4;
  return (b + 127) & ~size_t(127);
}

int gemv_stages(int K, bool need_f32) {
  const size_t act = gemv_act_bytes(K, need_f32);
  if (act >= (size_t)kSmemLimit) return 0;
  const int n = (int)((kSmemLimit - act) / kStageMax);
  return n < kMaxStages ? n : kMaxStages;
}

size_t gemv_smem_bytes(int K, bool need_f32) {
  return gemv_act_bytes(K, need_f32) + (size_t)gemv_stages(K, need_f32) * kStageMax;
}

size_t gemv_partial_floats(int64_t max_tiles) {
  return (size_t)max_tiles * kMaxKParts * 2 * kRPT;
}

cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t s, bool pdl) {
  const int sms = sm_count();
  Plan P;
  if (a.nseg < 1 || a.nseg > 4 || !make_plan(a, &P, sms)) return cudaErrorInvalidValue;
  P.stages = gemv_stages(a.K, P.need_f32 != 0);
  if (P.stages < 2) return cudaErrorInvalidValue;
  const size_t smem = gemv_smem_bytes(a.K, P.need_f32 != 0);
  const int grid = (int)(P.n_items < (int64_t)sms ? P.n_items : (int64_t)sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel, a, P);
}

}  // namespace rpgc
