// k_gemv.cu -- decode GEMV over raw ggml blocks (batch 1), sm_100a.
//
// Replaces the reference's fused dequant dot-row (src/matmul_avx2.cc:95-289,
// dispatched per row by QuantMatrix::MatVec/MatMulBatch, src/model.cc:23-69).
//
// Work split.  A row of K elements is cut into U = K/64 units of 64
// consecutive elements (a Q4_K group, a quarter of a Q6_K block, two Q8_0
// blocks).  Consumer thread t of a CTA owns unit u = t % U for the whole
// launch and is row slot s = t / U; S = floor(320 / U) slots work on S rows
// at a time, two rows per step so that one read of the activation serves two
// weight rows (a 128-bit shared load costs 3-4.5 SM cycles whatever its
// pattern, so activation reads, not weight reads, bound the inner loop).
// Each thread's partial sum of (row, unit) goes to shared memory; rows are
// summed over their U units in a fixed order once a chunk of stages is
// complete, so results are deterministic.
//
// Data path.  Every CTA owns a contiguous, balanced range of rows of each
// segment (no split along K).  Rows are contiguous in HBM, so one stage of
// the ring is ONE bulk async copy of m whole rows (16-24 KB: copies of that
// size stream at ~6 TB/s, 500-byte ones at ~2 TB/s).  A dedicated producer
// warp issues them with an evict-first L2 policy (issuing a bulk copy blocks
// the issuing thread for a time proportional to its size, so no consumer
// does it).  The first stages are issued before griddepcontrol.wait:
// weights do not depend on the previous kernel, so with programmatic
// dependent launch they stream in during its tail.  A CTA uses at most 112
// KB of shared memory and 2 x 352 x 88 registers fit an SM, so the next
// kernel's CTA can sit beside it.
//
// Arithmetic.  Activation groups of 32 get a power-of-two scale 2^(e-149)
// and a 24-bit integer copy held as three byte limbs A = 65536*A2 + 256*A1 +
// A0.  A block dot product is 3 dp4a per 4 weights with exact int32 partial
// sums, then the ggml scales are applied per sub-block in fp32:
//   Q4_K  s_g * (d*sc * S - dmin*m * sum(A))
//   Q6_K  s_g * d*sc * (S - 32 * sum(A))          (q stored as 0..63)
//   Q8_0  s_g * d * S
// The fixed-point rounding is 2^-24 of the group maximum, far inside the
// per-row gate max|d| / sum|a*w| <= 1e-5.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

constexpr int kCWarps = 10;                  // consumer warps
constexpr int kConsumers = kCWarps * 32;     // consumer threads
constexpr int kThreads = kConsumers + 32;    // + one producer warp
constexpr int kMaxStages = 6;
constexpr int kSmemLimit = 112 * 1024;       // leaves room for the next kernel's CTA
constexpr int kStageTarget = 24 * 1024;
constexpr int kRedBudget = 8 * 1024;         // partial sums of one reduction chunk (x2 buffers)

struct LSeg {      // logical segment: one matrix, or a SwiGLU (gate, up) pair
  int64_t rows;
  int32_t first;   // index into GemvArgs::seg
  int32_t pair;    // 1: seg[first] is the gate, seg[first + 1] the up matrix
  int32_t m;       // rows per stage (multiple of S)
  int32_t cs;      // stages per reduction chunk
};

struct Plan {
  LSeg ls[4];
  int32_t nls;
  int32_t U, S;          // units per row, row slots
  int32_t stages;        // ring depth
  int32_t stage_bytes;   // bytes per ring slot
  int32_t half_bytes;    // offset of the up matrix inside a slot
  int32_t red_floats;    // floats of the partial-sum buffer
  int32_t need_f32;
};

// ---------------------------------------------------------------- activation
// Fixed-point activation in shared memory, laid out so that the consumer
// threads of a warp (consecutive units) read consecutive 16-byte words:
// limb[(L * 4 + i) * U + u] holds words 4i..4i+3 of limb L (0: A2, 1: A1,
// 2: A0) of unit u, word j covering elements 4j..4j+3 of the unit.
struct ActS {
  const uint4* limb;
  const float* g;    // [2][U] group scales 2^(e-149) (0 for a flushed group)
  const float* gm;   // [2][U] Q4_K: g * sum(A) of each 32-element group
  const float* g6;   // [4][U] Q6_K: 32 * g * sum(A) of each 16-element sub-block
  const float* xf;   // [K] fp32 copy (F32 weights only)
  int U;
};

// Activation words 8h..8h+7 of the three limbs of unit u.
__device__ __forceinline__ void act_half(const ActS& A, int u, int h, uint32_t* a2, uint32_t* a1,
                                         uint32_t* a0) {
#pragma unroll
  for (int L = 0; L < 3; ++L) {
    const uint4 x = A.limb[(L * 4 + 2 * h) * A.U + u];
    const uint4 y = A.limb[(L * 4 + 2 * h + 1) * A.U + u];
    uint32_t* d = L == 0 ? a2 : (L == 1 ? a1 : a0);
    d[0] = x.x; d[1] = x.y; d[2] = x.z; d[3] = x.w;
    d[4] = y.x; d[5] = y.y; d[6] = y.z; d[7] = y.w;
  }
}

__device__ __forceinline__ float comb(int s2, int s1, int s0) {
  return (float)(s2 * 256 + s1) * 256.0f + (float)s0;
}

// fp16 in the low half of w -> fp32 (exact conversion).
__device__ __forceinline__ float half_lo(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
}

// N words starting at a 2-byte-aligned shared address, shifted right by
// `extra` more bits (0 or 4): N + 1 aligned loads and N funnel shifts.
template <int N>
__device__ __forceinline__ void ldw(const uint8_t* p, uint32_t extra, uint32_t* out) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 3) * 8 + extra;
  uint32_t prev = w[0];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t nx = w[j + 1];
    out[j] = __funnelshift_r(prev, nx, sh);
    prev = nx;
  }
}

// ------------------------------------------------------------ unit products
// Each computes one unit of R rows (R = 2: p0 and p1 share the activation reads).

// Q4_K: unit = group g (64 elements) of a 144-byte block (16-byte aligned).
// Low nibbles of qs[32g..32g+32) are elements 0..31, high nibbles 32..63; the
// high nibbles are used in place (16x) and the 1/16 is folded into the scale.
template <int R>
__device__ __forceinline__ void q4k_pair(const uint8_t* b0, const uint8_t* b1, int u, const ActS& A,
                                         float* y) {
  const int g = u & 3;
  const uint8_t* bp[2] = {b0, b1};
  uint4 hdr[2];
  uint32_t q[2][8];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    hdr[r] = *reinterpret_cast<const uint4*>(bp[r]);
    const uint4 qa = *reinterpret_cast<const uint4*>(bp[r] + 16 + 32 * g);
    const uint4 qb = *reinterpret_cast<const uint4*>(bp[r] + 32 + 32 * g);
    q[r][0] = qa.x; q[r][1] = qa.y; q[r][2] = qa.z; q[r][3] = qa.w;
    q[r][4] = qb.x; q[r][5] = qb.y; q[r][6] = qb.z; q[r][7] = qb.w;
  }
  float c[2][2];  // [row][sub-block] combined integer sums
#pragma unroll
  for (int h = 0; h < 2; ++h) {  // h = 0: low nibbles (elements 0..31), 1: high nibbles
    uint32_t a2[8], a1[8], a0[8];
    act_half(A, u, h, a2, a1, a0);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t w = q[r][j] & (h ? 0xF0F0F0F0u : 0x0F0F0F0Fu);
        s2 = dp4a_us(w, a2[j], s2);
        s1 = dp4a_uu(w, a1[j], s1);
        s0 = dp4a_uu(w, a0[j], s0);
      }
      c[r][h] = comb(s2, s1, s0);
    }
  }
  const float g0 = A.g[u], g1 = A.g[A.U + u] * 0.0625f;
  const float m0 = A.gm[u], m1 = A.gm[A.U + u];
  const uint32_t selP = (g & 1) ? 0x7632u : 0x5410u, selQ = (g & 1) ? 0x3232u : 0x1010u;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    // 6-bit (scale, min) of sub-blocks 2g and 2g+1 (ggml get_scale_min_k4) as
    // bytes [sc0, sc1, m0, m1]; the 12-byte scale field is hdr.y, hdr.z, hdr.w.
    // g < 2: bytes (2g, 2g+1) and (2g+4, 2g+5), low 6 bits.  g >= 2: low/high
    // nibbles of bytes 2g+4, 2g+5 with the top 2 bits of bytes 2g-4, 2g-3
    // (scales) and 2g, 2g+1 (mins).
    const uint32_t P = __byte_perm(hdr[r].y, hdr[r].z, selP);
    const uint32_t Q = __byte_perm(hdr[r].w, hdr[r].w, selQ);
    const uint32_t hiform = (Q & 0x00000F0Fu) | ((Q >> 4) & 0x0F0F0000u) | ((P >> 2) & 0x30303030u);
    const uint32_t SM = g >= 2 ? hiform : (P & 0x3F3F3F3Fu);
    const float d = half_lo(hdr[r].x), dmin = half_lo(hdr[r].x >> 16);
    y[r] = (d * (float)(SM & 0xFFu)) * (g0 * c[r][0]) - (dmin * (float)((SM >> 16) & 0xFFu)) * m0 +
           (d * (float)((SM >> 8) & 0xFFu)) * (g1 * c[r][1]) - (dmin * (float)(SM >> 24)) * m1;
  }
}

// Q6_K: unit v (0..3) of a 210-byte block (2-byte aligned) = elements
// [64v, 64v+64) = quadrants 2*odd and 2*odd+1 of half h = v >> 1, odd = v & 1:
// nibble 4*odd of ql[64h .. 64h+64), bit pairs 4*odd + (0, 2) of
// qh[32h .. 32h+32), int8 scales [4v, 4v+4), fp16 d at byte 208.
template <int R>
__device__ __forceinline__ void q6k_pair(const uint8_t* b0, const uint8_t* b1, int u, const ActS& A,
                                         float* y) {
  const int v = u & 3, h = v >> 1;
  const uint32_t ext = (uint32_t)(v & 1) * 4;
  const uint8_t* bp[2] = {b0, b1};
  uint32_t qh[2][8], sw[2], d2[2];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    ldw<8>(bp[r] + 128 + 32 * h, ext, qh[r]);
    ldw<1>(bp[r] + 192 + 4 * v, 0, &sw[r]);
    ldw<1>(bp[r] + 208, 0, &d2[r]);
  }
  float acc[2] = {0.0f, 0.0f};
#pragma unroll
  for (int part = 0; part < 2; ++part) {  // elements [32*part, 32*part + 32)
    uint32_t a2[8], a1[8], a0[8];
    act_half(A, u, part, a2, a1, a0);
    const float gp = A.g[part * A.U + u];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      uint32_t ql[8];
      ldw<8>(bp[r] + 64 * h + 32 * part, ext, ql);
      const float d = half_lo(d2[r]);
#pragma unroll
      for (int sb = 0; sb < 2; ++sb) {  // 16-element sub-block 2*part + sb
        int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = 4 * sb + jj;
          const uint32_t hb =
              part == 0 ? ((qh[r][j] << 4) & 0x30303030u) : ((qh[r][j] << 2) & 0x30303030u);
          const uint32_t q = (ql[j] & 0x0F0F0F0Fu) | hb;
          s2 = dp4a_us(q, a2[j], s2);
          s1 = dp4a_uu(q, a1[j], s1);
          s0 = dp4a_uu(q, a0[j], s0);
        }
        const int k = 2 * part + sb;
        const float sc = (float)(int)(int8_t)((sw[r] >> (8 * k)) & 0xFFu);
        acc[r] += (d * sc) * (gp * comb(s2, s1, s0) - A.g6[k * A.U + u]);
      }
    }
  }
  y[0] = acc[0];
  if (R == 2) y[1] = acc[1];
}

// Q8_0: unit = two 34-byte blocks (4-byte aligned): 17 words.
template <int R>
__device__ __forceinline__ void q8_0_pair(const uint8_t* b0, const uint8_t* b1, int u, const ActS& A,
                                          float* y) {
  const uint32_t* wp[2] = {reinterpret_cast<const uint32_t*>(b0), reinterpret_cast<const uint32_t*>(b1)};
  float acc[2] = {0.0f, 0.0f};
#pragma unroll
  for (int blk = 0; blk < 2; ++blk) {  // block 0: bytes 2..33, block 1: bytes 36..67
    uint32_t a2[8], a1[8], a0[8];
    act_half(A, u, blk, a2, a1, a0);
    const float gb = A.g[blk * A.U + u];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      uint32_t w[9];
#pragma unroll
      for (int j = 0; j < 9; ++j) w[j] = wp[r][8 * blk + j];
      int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t q = blk == 0 ? __funnelshift_r(w[j], w[j + 1], 16) : w[j + 1];
        s2 = dp4a_ss(q, a2[j], s2);
        s1 = dp4a_su(q, a1[j], s1);
        s0 = dp4a_su(q, a0[j], s0);
      }
      const float d = blk == 0 ? half_lo(w[0]) : half_lo(w[0] >> 16);
      acc[r] += d * (gb * comb(s2, s1, s0));
    }
  }
  y[0] = acc[0];
  if (R == 2) y[1] = acc[1];
}

// F32: unit = 64 floats, plain fp32 dot with the fp32 activation copy.
template <int R>
__device__ __forceinline__ void f32_pair(const uint8_t* b0, const uint8_t* b1, int u, const ActS& A,
                                         float* y) {
  const float4* w0 = reinterpret_cast<const float4*>(b0);
  const float4* w1 = reinterpret_cast<const float4*>(b1);
  const float4* x = reinterpret_cast<const float4*>(A.xf + 64 * u);
  float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 4
  for (int j = 0; j < 16; ++j) {
    const float4 v = x[j], p = w0[j], q = w1[j];
    s0 += p.x * v.x + p.y * v.y + p.z * v.z + p.w * v.w;
    if (R == 2) s1 += q.x * v.x + q.y * v.y + q.z * v.z + q.w * v.w;
  }
  y[0] = s0;
  if (R == 2) y[1] = s1;
}

// Type-mask bits: the block types a kernel instantiation handles.
constexpr uint32_t kMQ4K = 1, kMQ6K = 2, kMQ80 = 4, kMF32 = 8, kMAll = 15;

__host__ __device__ constexpr uint32_t type_bit(uint32_t type) {
  return type == kQ4_K ? kMQ4K : type == kQ6_K ? kMQ6K : type == kQ8_0 ? kMQ80 : type == kF32 ? kMF32 : 0;
}

// Unit u of R (1 or 2) rows.
template <int R, uint32_t TM>
__device__ __forceinline__ void unit_rows(uint32_t type, const uint8_t* p0, const uint8_t* p1, int u,
                                          const ActS& A, float* y) {
  if ((TM & kMQ4K) && type == kQ4_K) q4k_pair<R>(p0 + 144 * (u >> 2), p1 + 144 * (u >> 2), u, A, y);
  else if ((TM & kMQ6K) && type == kQ6_K) q6k_pair<R>(p0 + 210 * (u >> 2), p1 + 210 * (u >> 2), u, A, y);
  else if ((TM & kMQ80) && type == kQ8_0) q8_0_pair<R>(p0 + 68 * u, p1 + 68 * u, u, A, y);
  else if (TM & kMF32) f32_pair<R>(p0 + 256 * u, p1 + 256 * u, u, A, y);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

// ------------------------------------------------------------ stages
// The CTA's rows of logical segment i are [lo_i, hi_i) (balanced split of
// rows_i over the grid); they are streamed in stages of at most m_i rows.
__device__ __forceinline__ void cta_rows(const Plan& P, int ls, int64_t* lo, int64_t* hi) {
  const uint32_t rows = (uint32_t)P.ls[ls].rows;  // rows * grid < 2^32 (host check)
  *lo = rows * blockIdx.x / gridDim.x;
  *hi = rows * (blockIdx.x + 1) / gridDim.x;
}

__device__ __forceinline__ int count_stages(const Plan& P) {
  int n = 0;
  for (int i = 0; i < P.nls; ++i) {
    int64_t lo, hi;
    cta_rows(P, i, &lo, &hi);
    n += (int)((hi - lo + P.ls[i].m - 1) / P.ls[i].m);
  }
  return n;
}

// What the consumers need to know about a ring slot's current stage; written
// by the producer before it arms the slot's barrier.
struct StageDesc {
  int64_t r;      // first row
  int32_t n;      // rows
  int32_t ls;     // logical segment
  int32_t last;   // 1: last stage of its logical segment
  uint32_t off0;  // byte offset of row r inside the slot
  uint32_t off1;  // same for the up matrix of a pair
  int32_t pad;
};

// Producer-side walk over the stages (logical segment, row range).
struct Cursor {
  int ls;
  int64_t r, hi;
};

__device__ __forceinline__ void cursor_seek(const Plan& P, Cursor* c) {
  while (c->ls < P.nls && c->r >= c->hi) {
    if (++c->ls < P.nls) cta_rows(P, c->ls, &c->r, &c->hi);
  }
}

// Issue the next stage into `slot`: descriptor, barrier arming, one bulk copy
// of the rows (two for a pair), each from the 16-byte boundary at or below
// the first byte to the one at or above the last.
__device__ __forceinline__ void issue_next(const GemvArgs& A, const Plan& P, Cursor* c, uint8_t* dst,
                                           StageDesc* desc, uint64_t* bar, uint64_t pol) {
  const LSeg& L = P.ls[c->ls];
  const int64_t r = c->r;
  const int n = (int)(c->hi - r < L.m ? c->hi - r : L.m);
  const GemvSeg& G0 = A.seg[L.first];
  const uintptr_t s0 = reinterpret_cast<uintptr_t>(G0.w) + (uintptr_t)r * G0.row_bytes;
  const uintptr_t b0 = s0 & ~uintptr_t(15);
  const uint32_t n0 = (uint32_t)(((s0 + (uintptr_t)n * G0.row_bytes + 15) & ~uintptr_t(15)) - b0);
  uintptr_t b1 = 0, s1 = 0;
  uint32_t n1 = 0;
  if (L.pair) {
    const GemvSeg& G1 = A.seg[L.first + 1];
    s1 = reinterpret_cast<uintptr_t>(G1.w) + (uintptr_t)r * G1.row_bytes;
    b1 = s1 & ~uintptr_t(15);
    n1 = (uint32_t)(((s1 + (uintptr_t)n * G1.row_bytes + 15) & ~uintptr_t(15)) - b1);
  }
  StageDesc d;
  d.r = r;
  d.n = n;
  d.ls = c->ls;
  c->r += n;
  d.last = c->r >= c->hi;
  d.off0 = (uint32_t)(s0 - b0);
  d.off1 = (uint32_t)P.half_bytes + (uint32_t)(s1 - b1);
  d.pad = 0;
  *desc = d;
  cursor_seek(P, c);
  mbar_arrive_expect_tx(bar, n0 + n1);  // release: the descriptor is visible to the waiters
  bulk_g2s(dst, reinterpret_cast<const void*>(b0), n0, bar, pol);
  if (L.pair) bulk_g2s(dst + P.half_bytes, reinterpret_cast<const void*>(b1), n1, bar, pol);
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kConsumers) : "memory");
}

// Fixed-point limbs of NB consecutive-in-thread words (4 activation values
// each; word w of the thread is element block w = base + 320 * i).  Group
// maxima and sums come from the 8 lanes of a 32-element group (8
// consecutive lanes).  Straight-line: every word's shuffle chain is issued
// before any store, so the chains of different words overlap.
template <int NB>
__device__ __forceinline__ void quant_words(const float4 (&v)[NB], int w0, int NW, int U,
                                            uint32_t* limbw, float* ucon) {
  float gsc[NB], up[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    float a = fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w)));
    up[i] = a;
  }
#pragma unroll
  for (int n = 1; n <= 4; n <<= 1) {
#pragma unroll
    for (int i = 0; i < NB; ++i) up[i] = fmaxf(up[i], __shfl_xor_sync(0xffffffffu, up[i], n));
  }
  uint32_t l2[NB], l1[NB], l0[NB];
  int s16[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const uint32_t eb = (__float_as_uint(up[i]) >> 23) & 0xFFu;  // biased exponent of the group max
    const bool live = eb >= 30 && eb < 255;  // tinier groups contribute nothing
    // amax < 2^(eb-126): scaling by 2^(149-eb) keeps |q| < 2^23
    const float sc = live ? __uint_as_float((276u - eb) << 23) : 0.0f;
    gsc[i] = live ? __uint_as_float((eb - 22u) << 23) : 0.0f;  // 2^(eb-149)
    const int q0 = max(-8388607, min(8388607, __float2int_rn(v[i].x * sc)));
    const int q1 = max(-8388607, min(8388607, __float2int_rn(v[i].y * sc)));
    const int q2 = max(-8388607, min(8388607, __float2int_rn(v[i].z * sc)));
    const int q3 = max(-8388607, min(8388607, __float2int_rn(v[i].w * sc)));
    s16[i] = (q0 + q1) + (q2 + q3);
    const uint32_t a = (uint32_t)q0, b = (uint32_t)q1, c = (uint32_t)q2, d = (uint32_t)q3;
    l2[i] = __byte_perm(__byte_perm(a, b, 0x0062u), __byte_perm(c, d, 0x0062u), 0x5410u);
    l1[i] = __byte_perm(__byte_perm(a, b, 0x0051u), __byte_perm(c, d, 0x0051u), 0x5410u);
    l0[i] = __byte_perm(__byte_perm(a, b, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
  }
  int s32[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) s16[i] += __shfl_xor_sync(0xffffffffu, s16[i], 1);
#pragma unroll
  for (int i = 0; i < NB; ++i) s16[i] += __shfl_xor_sync(0xffffffffu, s16[i], 2);
#pragma unroll
  for (int i = 0; i < NB; ++i) s32[i] = s16[i] + __shfl_xor_sync(0xffffffffu, s16[i], 4);
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const int w = w0 + i * kConsumers;
    const int u = w >> 4, k = w & 15;  // unit, word in unit
    const int base = ((k >> 2) * U + u) * 4 + (k & 3);
    const bool in = w < NW;
    if (in) {
      limbw[base] = l2[i];
      limbw[base + 16 * U] = l1[i];
      limbw[base + 32 * U] = l0[i];
    }
    if (in && (k & 3) == 0) ucon[(4 + (k >> 2)) * U + u] = 32.0f * gsc[i] * (float)s16[i];
    if (in && (k & 7) == 0) {
      ucon[(k >> 3) * U + u] = gsc[i];
      ucon[(2 + (k >> 3)) * U + u] = gsc[i] * (float)s32[i];
    }
  }
}

// Activation prologue of the consumer threads: thread t handles the
// 4-element words w = t + 320 i (coalesced loads); the 8 lanes of a
// 32-element group are 8 consecutive lanes of one warp.  The RMSNorm gains
// are read before the grid-dependency wait (they do not depend on the
// previous kernel), x after it.  Returns false when the step is inactive.
__device__ __forceinline__ bool prologue(const GemvArgs& A, const Plan& P, int tid, int lane, int warp,
                                         double* dred, uint4* limb, float* ucon, float* xf) {
  constexpr int NB = 4;  // words per batch
  const int K = A.K, NW = K / 4, U = P.U;
  const float4* x4 = reinterpret_cast<const float4*>(A.x);
  const float4* n4 = reinterpret_cast<const float4*>(A.norm_w);
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  const bool norm = A.norm_w != nullptr;  // then NW <= 4 * 320 (host check): one batch
  float4 nv[NB];
  if (norm) {
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int w = tid + i * kConsumers;
      nv[i] = w < NW ? __ldg(n4 + w) : zero;
    }
  }
  grid_dep_wait();  // x (and *active) are written by the previous kernel
  if (A.active && __ldcg(A.active) == 0) return false;
  uint32_t* limbw = reinterpret_cast<uint32_t*>(limb);
  for (int b = 0; b < NW; b += NB * kConsumers) {  // uniform trip count
    float4 v[NB];
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int w = b + tid + i * kConsumers;
      v[i] = w < NW ? __ldcg(x4 + w) : zero;
    }
    if (norm) {  // RMSNorm scale of x (sum of squares in double)
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < NB; ++i)
        ss += (double)v[i].x * v[i].x + (double)v[i].y * v[i].y + (double)v[i].z * v[i].z +
              (double)v[i].w * v[i].w;
      ss = warp_sum(ss);
      if (lane == 0) dred[warp] = ss;
      consumer_sync();
      double tot = 0.0;
      for (int w = 0; w < kCWarps; ++w) tot += dred[w];
      const float nscale = (float)(1.0 / sqrt(tot / (double)K + (double)A.eps));
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        v[i].x = v[i].x * nscale * nv[i].x;
        v[i].y = v[i].y * nscale * nv[i].y;
        v[i].z = v[i].z * nscale * nv[i].z;
        v[i].w = v[i].w * nscale * nv[i].w;
      }
    }
    if (P.need_f32) {
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        const int w = b + tid + i * kConsumers;
        if (w < NW) reinterpret_cast<float4*>(xf)[w] = v[i];
      }
    }
    quant_words<NB>(v, b + tid, NW, U, limbw, ucon);
  }
  consumer_sync();  // limbs, per-unit constants (and the fp32 copy) are visible
  return true;
}

template <uint32_t TM>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ GemvArgs A,
                                                           const __grid_constant__ Plan P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = A.K, U = P.U, S = P.S, NS = P.stages;
  const int Ur = U | 1;  // row stride of the partial sums
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // ---- shared-memory carve-up (must match fixed_bytes())
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);              // [kMaxStages]
  uint64_t* empty = full + kMaxStages;                             // [kMaxStages]
  StageDesc* desc = reinterpret_cast<StageDesc*>(smem + 128);      // [kMaxStages]
  double* dred = reinterpret_cast<double*>(smem + 128 + 32 * kMaxStages);  // [16]
  float* ucon = reinterpret_cast<float*>(smem + 384);              // g[2U], gm[2U], g6[4U]
  uint4* limb = reinterpret_cast<uint4*>(smem + 384 + ((32 * U + 127) & ~127));  // [12][U]
  float* red = reinterpret_cast<float*>(limb + 12 * U);            // [2][red_floats]
  float* xf = red + 2 * P.red_floats;                              // [K] (F32 weights only)
  const uintptr_t sp = reinterpret_cast<uintptr_t>(xf + (P.need_f32 ? K : 0));
  uint8_t* stages = reinterpret_cast<uint8_t*>((sp + 127) & ~uintptr_t(127));

  const int n_stages = count_stages(P);
  if (n_stages == 0) {  // no rows for this CTA
    grid_dep_launch();
    return;
  }
  Cursor cur;
  if (tid == kConsumers) {  // producer lane: barriers, first stages
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCWarps);
    }
    fence_barrier_init();
    const uint64_t pol = policy_evict_first();
    cur.ls = 0;
    cta_rows(P, 0, &cur.r, &cur.hi);
    cursor_seek(P, &cur);
    for (int i = 0; i < NS && i < n_stages; ++i)
      issue_next(A, P, &cur, stages + (size_t)i * P.stage_bytes, &desc[i], &full[i], pol);
  }
  grid_dep_launch();  // the next kernel may start its own weight prefetch
  __syncthreads();

  if (warp == kCWarps) {
    // ============================================================ producer
    if (lane != 0) return;
    grid_dep_wait();  // *active is written by the previous kernel
    if (A.active && __ldcg(A.active) == 0) {  // drain the copies in flight, then leave
      for (int i = 0; i < NS && i < n_stages; ++i) mbar_wait(&full[i], 0, A.err);
      return;
    }
    const uint64_t pol = policy_evict_first();
    for (int it = NS; it < n_stages; ++it) {
      const int slot = it % NS;
      mbar_wait(&empty[slot], (uint32_t)(it / NS - 1) & 1u, A.err);
      issue_next(A, P, &cur, stages + (size_t)slot * P.stage_bytes, &desc[slot], &full[slot], pol);
    }
    return;
  }

  // ============================================================== consumers
  if (!prologue(A, P, tid, lane, warp, dred, limb, ucon, xf)) return;

  ActS act;
  act.limb = limb;
  act.g = ucon;
  act.gm = ucon + 2 * U;
  act.g6 = ucon + 4 * U;
  act.xf = xf;
  act.U = U;
  const int u = tid % U, s = tid / U;
  const bool busy = s < S;

  // ---- main loop over the ring
  int chunk_it0 = 0;      // first stage of the current reduction chunk
  int64_t chunk_r0 = 0;   // its first row
  int cbuf = 0;           // partial-sum buffer of the chunk
  for (int it = 0; it < n_stages; ++it) {
    const int slot = it % NS;
    mbar_wait(&full[slot], (uint32_t)(it / NS) & 1u, A.err);
    const StageDesc d = desc[slot];
    const LSeg& L = P.ls[d.ls];
    const GemvSeg& G = A.seg[L.first];
    const int rb = (int)G.row_bytes;
    const uint32_t type = G.type;
    if (it == chunk_it0) chunk_r0 = d.r;
    const int jr0 = (it - chunk_it0) * L.m;  // row of this stage inside the chunk
    const int ck_rows = L.cs * L.m;          // row capacity of a chunk
    float* rbuf = red + cbuf * P.red_floats;
    const uint8_t* sb = stages + (size_t)slot * P.stage_bytes;
    if (busy) {
      float y[2];
      const uint8_t* base0 = sb + d.off0;
      if (L.pair) {  // gate and up rows j share the activation
        const uint8_t* base1 = sb + d.off1;
        for (int j = s; j < d.n; j += S) {
          unit_rows<2, TM>(type, base0 + j * rb, base1 + j * rb, u, act, y);
          rbuf[(jr0 + j) * Ur + u] = y[0];
          rbuf[(ck_rows + jr0 + j) * Ur + u] = y[1];
        }
      } else {  // rows j and j + S together
        int j = s;
        for (; j + S < d.n; j += 2 * S) {
          unit_rows<2, TM>(type, base0 + j * rb, base0 + (j + S) * rb, u, act, y);
          rbuf[(jr0 + j) * Ur + u] = y[0];
          rbuf[(jr0 + j + S) * Ur + u] = y[1];
        }
        if (j < d.n) {  // an odd row out
          unit_rows<1, TM>(type, base0 + j * rb, base0 + j * rb, u, act, y);
          rbuf[(jr0 + j) * Ur + u] = y[0];
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);  // the slot may be refilled
    if (!d.last && it + 1 - chunk_it0 < L.cs) continue;
    // ---- chunk complete: every row total is summed by 4 threads (units
    // u = q mod 4) whose results are added by two shuffles; for a pair the
    // gate and up totals of a row sit in 8 consecutive lanes.  Fixed order,
    // so deterministic.  The other buffer takes the next chunk, and this one
    // is not written again before the next chunk's barrier.
    consumer_sync();
    const int rows = jr0 + d.n;
    const int nsum = rows * (L.pair + 1);
    for (int b0 = 0; b0 < 4 * nsum; b0 += kConsumers) {  // warp-uniform trip count
      const int idx = b0 + tid, q = idx & 3, sid = idx >> 2;
      const int j = L.pair ? sid >> 1 : sid, h = L.pair ? sid & 1 : 0;
      float t = 0.0f;
      if (sid < nsum) {
        const float* p = rbuf + (h * ck_rows + j) * Ur;
        for (int v = q; v < U; v += 4) t += p[v];
      }
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      const float other = __shfl_xor_sync(0xffffffffu, t, 4);  // up total for a pair's gate lane
      if (sid < nsum && q == 0 && h == 0) {
        const int64_t row = chunk_r0 + j;
        if (L.pair) A.seg[L.first + 1].out[row] = silu_mul(t, other);
        else if (G.mode == kAdd) G.out[row] += t;
        else G.out[row] = t;
      }
    }
    chunk_it0 = it + 1;
    cbuf ^= 1;
  }
}

// Work decomposition shared by the launcher and the kernel.
bool make_plan(const GemvArgs& a, Plan* P) {
  if (a.nseg < 1 || a.nseg > 4 || a.K <= 0 || a.K % 64 != 0) return false;
  if (a.norm_w && a.K > 16 * kConsumers) return false;  // gains preloaded: one batch of words
  const int U = a.K / 64;
  if (U > kConsumers) return false;
  P->U = U;
  P->S = kConsumers / U;
  P->need_f32 = 0;
  P->nls = 0;
  int stage_bytes = 0, half_bytes = 0, red = 0;
  for (int i = 0; i < a.nseg; ++i) {
    const GemvSeg& G = a.seg[i];
    int be, bb;
    switch (G.type) {
      case kQ4_K: be = 256; bb = 144; break;
      case kQ6_K: be = 256; bb = 210; break;
      case kQ8_0: be = 32; bb = 34; break;
      case kF32: be = 32; bb = 128; P->need_f32 = 1; break;
      default: return false;
    }
    if (a.K % be != 0 || (int64_t)(a.K / be) * bb != G.row_bytes) return false;
    if (reinterpret_cast<uintptr_t>(G.w) & 15) return false;  // bulk copies need 16 B
    if (G.rows <= 0 || G.rows > (int64_t)(0xFFFFFFFFu / 1024)) return false;
    const bool up_of_pair = i > 0 && a.seg[i - 1].mode == kSwiGLU;
    if (up_of_pair) {
      if (G.rows != a.seg[i - 1].rows || G.type != a.seg[i - 1].type) return false;
      continue;
    }
    LSeg& L = P->ls[P->nls++];
    L.rows = G.rows;
    L.first = i;
    L.pair = G.mode == kSwiGLU ? 1 : 0;
    const int64_t per_round = (int64_t)P->S * G.row_bytes * (L.pair + 1);
    int64_t rounds = kStageTarget / per_round;
    if (rounds < 1) rounds = 1;
    L.m = (int32_t)(rounds * P->S);
    const int64_t slot = ((int64_t)L.m * G.row_bytes + 32 + 127) & ~int64_t(127);
    if (slot > kSmemLimit / 2) return false;
    if (L.pair) half_bytes = half_bytes > (int)slot ? half_bytes : (int)slot;
    const int need = (int)slot * (L.pair + 1);
    stage_bytes = stage_bytes > need ? stage_bytes : need;
    const int per_stage = L.m * (U | 1) * (L.pair + 1);  // partial sums of one stage
    int cs = kRedBudget / (4 * per_stage);
    if (cs < 1) cs = 1;
    L.cs = cs;
    red = red > cs * per_stage ? red : cs * per_stage;
  }
  if (a.seg[a.nseg - 1].mode == kSwiGLU) return false;
  P->stage_bytes = stage_bytes;
  P->half_bytes = half_bytes;
  P->red_floats = red;
  return true;
}

size_t fixed_bytes(const Plan& P, int K) {
  const size_t b = 384 + (((size_t)32 * P.U + 127) & ~size_t(127)) + (size_t)12 * 16 * P.U +
                   (size_t)2 * P.red_floats * 4 + (P.need_f32 ? (size_t)K * 4 : 0);
  return (b + 127) & ~size_t(127);
}

// Kernel instantiations by type mix.
template <uint32_t TM>
void configure(int dev) {
  static bool done[64] = {false};
  if (dev < 0 || dev >= 64 || done[dev]) return;
  cudaFuncSetAttribute(gemv_kernel<TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  // the largest shared-memory carveout, so that two CTAs (this kernel's and
  // the next kernel's) fit on an SM at once
  cudaFuncSetAttribute(gemv_kernel<TM>, cudaFuncAttributePreferredSharedMemoryCarveout,
                       cudaSharedmemCarveoutMaxShared);
  done[dev] = true;
}

int sm_count(int dev) {
  static int sms[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = n > 0 && n <= 1024 ? n : 148;
  }
  return sms[dev];
}

template <uint32_t TM>
cudaError_t launch_tm(const GemvArgs& a, const Plan& P, cudaLaunchConfig_t* cfg, int dev) {
  configure<TM>(dev);
  const cudaError_t e_ = cudaLaunchKernelEx(cfg, gemv_kernel<TM>, a, P);
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

}  // namespace

cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t s, bool pdl) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = sm_count(dev);
  Plan P;
  if (!make_plan(a, &P)) return cudaErrorInvalidValue;
  const size_t fixed = fixed_bytes(P, a.K);
  if (fixed + 2 * (size_t)P.stage_bytes > (size_t)kSmemLimit) return cudaErrorInvalidValue;
  const int ns = (int)((kSmemLimit - fixed) / P.stage_bytes);
  P.stages = ns < kMaxStages ? ns : kMaxStages;
  const size_t smem = fixed + (size_t)P.stages * P.stage_bytes;
  int64_t max_rows = 0;
  uint32_t mask = 0;
  for (int i = 0; i < P.nls; ++i) max_rows = P.ls[i].rows > max_rows ? P.ls[i].rows : max_rows;
  for (int i = 0; i < a.nseg; ++i) mask |= type_bit(a.seg[i].type);
  const int grid = (int)(max_rows < (int64_t)sms ? max_rows : (int64_t)sms);
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
  // One instantiation serves every launch of a model's decode step (the
  // K-quant mix, or Q8_0): consecutive kernels then run the same code, which
  // stays in the instruction caches.
  if ((mask & ~(kMQ4K | kMQ6K)) == 0) return launch_tm<kMQ4K | kMQ6K>(a, P, &cfg, dev);
  if (mask == kMQ80) return launch_tm<kMQ80>(a, P, &cfg, dev);
  return launch_tm<kMAll>(a, P, &cfg, dev);
}

}  // namespace rpgc
