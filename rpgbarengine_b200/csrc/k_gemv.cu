// k_gemv.cu -- decode GEMV over raw ggml blocks (batch 1), sm_100a.
//
// Replaces the reference's fused dequant dot-row (src/matmul_avx2.cc:95-289,
// dispatched per row by QuantMatrix::MatVec/MatMulBatch, src/model.cc:23-69).
//
// Work split.  A row of K elements is cut into U = K/64 units.  Unit u covers
// half-block hb = u/2 (elements [128 hb, 128 hb + 128)) and within it the
// four runs of 16 elements 128 hb + 32 j + 16 (u & 1) + [0, 16), j = 0..3.
// This interleaved shape reads every weight byte of a unit once for all three
// block formats: in a Q4_K block it is 16 bytes of quants of group 2h and 16
// of group 2h+1 (both nibbles used); in Q6_K 16 bytes of each of the two ql
// planes and 16 of qh (all bits used); in Q8_0 16 quants of four blocks.
// Consumer thread t of a CTA owns unit u = t % U for the whole launch and is
// row slot s = t / U (S slots).  Its unit of the activation, in fixed point,
// lives in 48 registers, so the inner loop reads only weights from shared
// memory.  Each thread's partial sum of (row, unit) goes to shared memory;
// rows are summed over their U units in a fixed order once a chunk of stages
// is complete, so results are deterministic.
//
// Data path.  Every CTA (one per SM) owns a contiguous, balanced range of rows
// of each segment (no split along K).  Rows are contiguous in HBM, so one
// stage of the ring is ONE bulk async copy of m whole rows (~32 KB: copies of
// that size stream at ~6 TB/s, 500-byte ones at ~2 TB/s).  A producer warp
// issues them (issuing a bulk copy blocks the issuing thread for a time
// proportional to its size, so no consumer does it).  The first stages are
// issued before griddepcontrol.wait: weights do not depend on the previous
// kernel.  Once its last stage is issued, the producer prefetches into L2 the
// first rows that the same CTA index of the NEXT matrix-vector launch will
// read, so that the next kernel's first stages come from L2.
//
// Arithmetic.  The 64 activation values of a unit (RMSNorm gains applied)
// share a power-of-two scale 2^(e-148) and become integers below 2^22 in
// magnitude held as three byte limbs A = 65536*A2 + 256*A1 + A0.  A run of 16 is 3 x 4 dp4a
// with exact int32 partial sums; the ggml scales are applied per run in fp32:
//   Q4_K  g * d*sc * S - dmin*m * g*sum(A)
//   Q6_K  d*sc * (g*S - 32 * g*sum(A))          (q stored as 0..63)
//   Q8_0  g * d * S
// The fixed-point rounding is 2^-23 of the unit maximum, far inside the
// per-row gate max|d| / sum|a*w| <= 1e-5.  The RMSNorm factor 1/rms is a
// scalar of the whole vector, so it multiplies the row totals at the end
// (y = W (x * gain) / rms) instead of the inputs: no barrier waits for the
// sum of squares before quantisation.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

#ifndef RPGC_GEMV_CWARPS
#define RPGC_GEMV_CWARPS 15
#endif
#ifndef RPGC_GEMV_STAGE_KB
#define RPGC_GEMV_STAGE_KB 32
#endif
#ifndef RPGC_GEMV_PRE
#define RPGC_GEMV_PRE 8
#endif
#ifndef RPGC_GEMV_XGATE
#define RPGC_GEMV_XGATE 0
#endif
constexpr int kMaxCWarps = RPGC_GEMV_CWARPS;      // consumer warps at most
constexpr int kMaxConsumers = kMaxCWarps * 32;    // 480
constexpr int kMaxThreads = kMaxConsumers + 32;   // + one producer warp
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 200 * 1024;            // one CTA per SM
constexpr int kStageTarget = RPGC_GEMV_STAGE_KB * 1024;

constexpr int kPreStages = RPGC_GEMV_PRE;         // stages issued before the dependency wait
constexpr bool kXGate = RPGC_GEMV_XGATE != 0;     // the other first stages wait for x
constexpr int kRedBudget = 16 * 1024;             // partial sums of one reduction chunk (x2 buffers)

struct LSeg {      // logical segment: one matrix, or a SwiGLU (gate, up) pair
  int64_t rows;
  int32_t first;   // index into GemvArgs::seg
  int32_t pair;    // 1: seg[first] is the gate, seg[first + 1] the up matrix
  int32_t m;       // rows per stage (multiple of S; of 2S unless a pair)
  int32_t cs;      // stages per reduction chunk
};

struct Plan {
  LSeg ls[4];
  int32_t nls;
  int32_t U, S, NC;      // units per row, row slots, consumer threads
  int32_t stages;        // ring depth
  int32_t stage_bytes;   // bytes per ring slot
  int32_t half_bytes;    // offset of the up matrix inside a slot
  int32_t red_floats;    // floats of the partial-sum buffer
  int32_t need_f32;
};

// ---------------------------------------------------------------- activation
// One unit of the activation in registers: limb L (0: A2 signed, 1: A1,
// 2: A0), word 4j + k = elements 4k..4k+3 of run j.
struct ActR {
  uint32_t a[3][16];
  float g;       // unit scale 2^(e-148) (0 for a flushed unit)
  float ga[4];   // g * sum(A) of run j
};

// fp16 in the low half of w -> fp32 (exact conversion).
__device__ __forceinline__ float half_lo(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
}

// Byte j of w as a float (exact): the byte under the exponent of 2^23.
template <int J>
__device__ __forceinline__ float byte_f(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + J)) - 8388608.0f;
}

// Shared-memory loads on 32-bit shared addresses (volatile: they stay after
// the mbarrier wait that makes the stage's bytes visible).
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}

// N words at a 2-byte-aligned shared address given as its 4-byte-aligned
// base al and the bit shift sh (0 or 16): N + 1 loads, N funnel shifts.
template <int N>
__device__ __forceinline__ void ldw(uint32_t al, uint32_t sh, uint32_t* out) {
  uint32_t w[N + 1];
#pragma unroll
  for (int j = 0; j <= N; ++j) w[j] = lds32(al + 4 * j);
#pragma unroll
  for (int j = 0; j < N; ++j) out[j] = __funnelshift_r(w[j], w[j + 1], sh);
}

__device__ __forceinline__ float comb_f(int s2, int s1, int s0) {
  return (float)s2 * 65536.0f + (float)((s1 << 8) + s0);
}

// Per-thread constants of its unit u: byte offsets inside a row.
struct UnitOff {
  uint32_t q4_hd, q4_qa, q4_qb;     // Q4_K: header, quants of groups 2h and 2h+1
  uint32_t q6_blk, q6_qa, q6_qb, q6_qh, q6_sc;  // Q6_K: block, offsets inside it
  uint32_t q8_blk;                  // Q8_0: first of the four blocks (+ 2 + 16 i)
  uint32_t hh, ip;
};

__device__ __forceinline__ UnitOff unit_offsets(int u) {
  UnitOff o;
  o.hh = (uint32_t)(u >> 1) & 1u;
  o.ip = (uint32_t)u & 1u;
  o.q4_hd = 144u * (uint32_t)(u >> 2);
  o.q4_qa = o.q4_hd + 16u + 64u * o.hh + 16u * o.ip;
  o.q4_qb = o.q4_qa + 32u;
  o.q6_blk = 210u * (uint32_t)(u >> 2);
  o.q6_qa = 64u * o.hh + 16u * o.ip;
  o.q6_qb = o.q6_qa + 32u;
  o.q6_qh = 128u + 32u * o.hh + 16u * o.ip;
  o.q6_sc = 192u + 8u * o.hh;
  o.q8_blk = 34u * 4u * (uint32_t)(u >> 1) + 2u + 16u * o.ip;
  return o;
}

// ------------------------------------------------------------ unit products
// Each computes unit u of R rows starting at shared addresses ba[r].

// Q4_K: block of 144 bytes (16-byte aligned): d, dmin, 12 scale bytes, 128
// quant bytes.  Runs 0/1 are the low/high nibbles of quants 64h + 16i .. +16
// (sub-blocks 4h, 4h+1), runs 2/3 those of 64h + 32 + 16i (4h+2, 4h+3).  A
// high nibble is used in place (16 q, still a byte), so its sums are 16x and
// the 1/16 is folded into the scale.
template <int R>
__device__ __forceinline__ void q4k_unit(const uint32_t* ba, const UnitOff& O, const ActR& A, float* y) {
  uint4 hd[R], qa[R], qb[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    hd[r] = lds128(ba[r] + O.q4_hd);
    qa[r] = lds128(ba[r] + O.q4_qa);
    qb[r] = lds128(ba[r] + O.q4_qb);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint32_t qw[8] = {qa[r].x, qa[r].y, qa[r].z, qa[r].w, qb[r].x, qb[r].y, qb[r].z, qb[r].w};
    float S[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t v = qw[4 * (j >> 1) + k];
        const uint32_t w = (j & 1) ? (v & 0xF0F0F0F0u) : (v & 0x0F0F0F0Fu);
        s2 = dp4a_us(w, A.a[0][4 * j + k], s2);
        s1 = dp4a_uu(w, A.a[1][4 * j + k], s1);
        s0 = dp4a_uu(w, A.a[2][4 * j + k], s0);
      }
      S[j] = comb_f(s2, s1, s0);  // 16x for the high-nibble runs
    }
    // 6-bit (scale, min) of sub-blocks 4h..4h+3 (ggml get_scale_min_k4) as
    // the bytes of SC and MN; the scale field is hd.y (bytes 0-3), hd.z
    // (4-7), hd.w (8-11).
    const uint4 h = hd[r];
    const uint32_t SC = O.hh ? ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)) : (h.y & 0x3F3F3F3Fu);
    const uint32_t MN = O.hh ? (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3F3F3F3Fu);
    float t1 = byte_f<0>(SC) * S[0];
    t1 = fmaf(byte_f<1>(SC) * 0.0625f, S[1], t1);
    t1 = fmaf(byte_f<2>(SC), S[2], t1);
    t1 = fmaf(byte_f<3>(SC) * 0.0625f, S[3], t1);
    float t2 = byte_f<0>(MN) * A.ga[0];
    t2 = fmaf(byte_f<1>(MN), A.ga[1], t2);
    t2 = fmaf(byte_f<2>(MN), A.ga[2], t2);
    t2 = fmaf(byte_f<3>(MN), A.ga[3], t2);
    y[r] = half_lo(h.x) * (A.g * t1) - half_lo(h.x >> 16) * t2;
  }
}

// Q6_K: block of 210 bytes (2-byte aligned): ql[128], qh[64], int8 sc[16],
// fp16 d.  Half h, i = u & 1: QA = ql[64h + 16i .. +16], QB = ql[64h + 32 +
// 16i .. +16], QH = qh[32h + 16i .. +16].  Run j: low (j < 2) or high nibble
// of QA (even j) / QB (odd j), bits 2j, 2j+1 of QH, scale sc[8h + i + 2j].
// All of a unit's fields sit at multiples of 4 bytes from each other, so one
// funnel shift amount serves every word.
template <int R>
__device__ __forceinline__ void q6k_unit(const uint32_t* ba, const UnitOff& O, const ActR& A, float* y) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint32_t p = ba[r] + O.q6_blk;
    const uint32_t al = p & ~3u, sh = (p & 3u) * 8u;
    uint32_t qa[4], qb[4], qh[4], sw[2];
    ldw<4>(al + O.q6_qa, sh, qa);
    ldw<4>(al + O.q6_qb, sh, qb);
    ldw<4>(al + O.q6_qh, sh, qh);
    ldw<2>(al + O.q6_sc, sh, sw);
    const float d = half_lo(lds16(p + 208u));
    const uint32_t ssh = 8u * O.ip;
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t b = (j & 1) ? qb[k] : qa[k];
        const uint32_t lo = (j >> 1) ? ((b >> 4) & 0x0F0F0F0Fu) : (b & 0x0F0F0F0Fu);
        const uint32_t hi = j == 0 ? (qh[k] << 4) : j == 1 ? (qh[k] << 2) : j == 2 ? qh[k] : (qh[k] >> 2);
        const uint32_t w = lo | (hi & 0x30303030u);
        s2 = dp4a_us(w, A.a[0][4 * j + k], s2);
        s1 = dp4a_uu(w, A.a[1][4 * j + k], s1);
        s0 = dp4a_uu(w, A.a[2][4 * j + k], s0);
      }
      const float t = fmaf(comb_f(s2, s1, s0), A.g, -32.0f * A.ga[j]);
      const float sc = (float)(int)(int8_t)((sw[j >> 1] >> (16 * (j & 1) + ssh)) & 0xFFu);
      acc = fmaf(sc, t, acc);
    }
    y[r] = d * acc;
  }
}

// Q8_0: run j is quants 16i .. 16i+16 of block 4 hb + j (34-byte blocks,
// 2-byte aligned; the four runs are 34 bytes apart, so their shifts differ).
template <int R>
__device__ __forceinline__ void q8_0_unit(const uint32_t* ba, const UnitOff& O, const ActR& A, float* y) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t p = ba[r] + O.q8_blk + 34u * j;  // first quant of the run
      uint32_t w[4];
      ldw<4>(p & ~3u, (p & 3u) * 8u, w);
      const float d = half_lo(lds16(p - 2u - 16u * O.ip));
      int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s2 = dp4a_ss(w[k], A.a[0][4 * j + k], s2);
        s1 = dp4a_su(w[k], A.a[1][4 * j + k], s1);
        s0 = dp4a_su(w[k], A.a[2][4 * j + k], s0);
      }
      acc = fmaf(d, comb_f(s2, s1, s0), acc);
    }
    y[r] = A.g * acc;
  }
}

// F32: plain fp32 dot of the unit's 64 floats with the fp32 activation copy.
template <int R>
__device__ __forceinline__ void f32_unit(const uint32_t* ba, int u, const float* xf, float* y) {
  const int e0 = 128 * (u >> 1) + 16 * (u & 1);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4* x4 = reinterpret_cast<const float4*>(xf + e0 + 32 * j);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 a = lds128(ba[r] + 4u * (uint32_t)(e0 + 32 * j + 4 * k));
        const float4 b = x4[k];
        acc += __uint_as_float(a.x) * b.x + __uint_as_float(a.y) * b.y + __uint_as_float(a.z) * b.z +
               __uint_as_float(a.w) * b.w;
      }
    }
    y[r] = acc;
  }
}

// Type-mask bits: the block types a kernel instantiation handles.
constexpr uint32_t kMQ4K = 1, kMQ6K = 2, kMQ80 = 4, kMF32 = 8, kMAll = 15;

__host__ __device__ constexpr uint32_t type_bit(uint32_t type) {
  return type == kQ4_K ? kMQ4K : type == kQ6_K ? kMQ6K : type == kQ8_0 ? kMQ80 : type == kF32 ? kMF32 : 0;
}

// Unit u of R (1 or 2) rows.
template <int R, uint32_t TM>
__device__ __forceinline__ void unit_rows(uint32_t type, const uint32_t* ba, int u, const UnitOff& O,
                                          const ActR& A, const float* xf, float* y) {
  if ((TM & kMQ4K) && type == kQ4_K) q4k_unit<R>(ba, O, A, y);
  else if ((TM & kMQ6K) && type == kQ6_K) q6k_unit<R>(ba, O, A, y);
  else if ((TM & kMQ80) && type == kQ8_0) q8_0_unit<R>(ba, O, A, y);
  else if (TM & kMF32) f32_unit<R>(ba, u, xf, y);
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
static_assert(sizeof(StageDesc) == 32 && kMaxStages * 16 <= 128 && kMaxStages * 32 <= 256,
              "shared-memory header: barriers [0, 128), descriptors [128, 384)");

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

// L2 prefetch of the first rows the same CTA index of the next launch reads.
__device__ __forceinline__ void prefetch_next(const GemvArgs& A) {
#pragma unroll 1
  for (int i = 0; i < A.npf; ++i) {
    const GemvPrefetch& F = A.pf[i];
    const uint32_t rows = (uint32_t)F.rows, rb = (uint32_t)F.row_bytes;  // host-checked ranges
    const uint32_t lo = rows * blockIdx.x / gridDim.x, hi = rows * (blockIdx.x + 1) / gridDim.x;
    if (hi <= lo) continue;
    const uint32_t bytes = min((hi - lo) * rb, (uint32_t)A.pf_bytes);
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(F.w) + (uintptr_t)lo * rb;
    const uintptr_t b0 = s0 & ~uintptr_t(15);
    const uint32_t n = ((uint32_t)(s0 - b0) + bytes + 15u) & ~15u;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b0), "r"(n) : "memory");
  }
}

// 16-byte asynchronous global -> shared copy through L2 (not L1: the source
// may have been written by the previous kernel).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void consumer_sync(int nc) {
  asm volatile("bar.sync 1, %0;" ::"r"(nc) : "memory");
}

// Quantise item i = elements [8i, 8i+8) (half-block hb = i >> 4, run
// j = (i >> 2) & 3, unit u = 2 hb + ((i >> 1) & 1), words 2t, 2t+1 of the
// run, t = i & 1).  The eight items of a unit sit on lanes that differ in
// bits 0, 2 and 3 of the item index (the item index and the lane agree mod
// 32), so the unit maximum is three xor-shuffles away and a run's sum one.
// Rounding to an integer is one multiply-add: v * 2^(148-e) + 1.5 * 2^23
// lies in [2^23, 2^24], where floats are the integers, so the low bits of
// the sum are round(v * 2^(148-e)) + 2^22.
__device__ __forceinline__ void quantize_item(float4 v0, float4 v1, int i, bool in, int U, uint4* lim,
                                              float* ucon) {
  float a = fmaxf(fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v0.z), fabsf(v0.w))),
                  fmaxf(fmaxf(fabsf(v1.x), fabsf(v1.y)), fmaxf(fabsf(v1.z), fabsf(v1.w))));
  a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
  a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
  a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 8));
  const uint32_t eb = (__float_as_uint(a) >> 23) & 0xFFu;  // biased exponent of the unit max
  const bool live = eb >= 30 && eb < 255;  // tinier units contribute nothing
  // amax < 2^(eb-126): scaling by 2^(148-eb) keeps |v * sc| < 2^22
  const float sc = live ? __uint_as_float((275u - eb) << 23) : 0.0f;
  const float gsc = live ? __uint_as_float((eb - 21u) << 23) : 0.0f;  // 2^(eb-148)
  const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  uint32_t q[8];
  int s = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    q[k] = __float_as_uint(fmaf(vv[k], sc, 12582912.0f)) - 0x4B400000u;
    s += (int)q[k];
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);  // run sum (16 elements)
  uint32_t l2[2], l1[2], l0[2];
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const uint32_t a0 = q[4 * w], a1 = q[4 * w + 1], a2 = q[4 * w + 2], a3 = q[4 * w + 3];
    const uint32_t X = __byte_perm(a0, a1, 0x5140u), Y = __byte_perm(a2, a3, 0x5140u);
    l0[w] = __byte_perm(X, Y, 0x5410u);
    l1[w] = __byte_perm(X, Y, 0x7632u);
    l2[w] = __byte_perm(__byte_perm(a0, a1, 0x0062u), __byte_perm(a2, a3, 0x0062u), 0x5410u);
  }
  if (in) {
    const int j = (i >> 2) & 3, u = 2 * (i >> 4) + ((i >> 1) & 1), t = i & 1;
    reinterpret_cast<uint2*>(lim + (0 * 4 + j) * U + u)[t] = make_uint2(l2[0], l2[1]);
    reinterpret_cast<uint2*>(lim + (1 * 4 + j) * U + u)[t] = make_uint2(l1[0], l1[1]);
    reinterpret_cast<uint2*>(lim + (2 * 4 + j) * U + u)[t] = make_uint2(l0[0], l0[1]);
    if (t == 0) ucon[(1 + j) * U + u] = gsc * (float)s;
    if (t == 0 && j == 0) ucon[u] = gsc;
  }
}

// Activation prologue of the consumer threads.  x (and the RMSNorm gains,
// before the grid-dependency wait: they do not depend on the previous
// kernel) are staged in shared memory by 16-byte asynchronous copies, so all
// loads are in flight at once; then thread t quantises items t + NC b.
// Returns false when the step is inactive.
__device__ __forceinline__ bool prologue(const GemvArgs& A, const Plan& P, int tid, int lane, int warp,
                                         double* dred, uint4* lim, float* ucon, float* xf,
                                         float4* stage_x, uint64_t* xready) {
  const int K = A.K, NI = K / 8, NC = P.NC, U = P.U, NW = K / 4;
  const bool norm = A.norm_w != nullptr;
  float4* xs = stage_x;
  float4* gs = stage_x + NW;  // gains (norm only)
  if (norm) {
#pragma unroll 1
    for (int w = tid; w < NW; w += NC) cp_async16(gs + w, reinterpret_cast<const float4*>(A.norm_w) + w);
  }
  grid_dep_wait();  // x (and *active) are written by the previous kernel
  grid_dep_launch();
  if (A.active && __ldcg(A.active) == 0) {
    cp_async_wait_all();
    return false;
  }
#pragma unroll 1
  for (int w = tid; w < NW; w += NC) cp_async16(xs + w, reinterpret_cast<const float4*>(A.x) + w);
  cp_async_wait_all();
  consumer_sync(NC);
  if (tid == 0) mbar_arrive(xready);  // the producer may issue the remaining first stages
  double ss = 0.0;
#pragma unroll 1
  for (int b = 0; b < NI; b += NC) {  // uniform trip count
    const int i = b + tid;
    const bool in = i < NI;
    float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
    if (in) {
      v0 = xs[2 * i];
      v1 = xs[2 * i + 1];
      if (norm) {
        ss += (double)v0.x * v0.x + (double)v0.y * v0.y + (double)v0.z * v0.z + (double)v0.w * v0.w +
              (double)v1.x * v1.x + (double)v1.y * v1.y + (double)v1.z * v1.z + (double)v1.w * v1.w;
        const float4 g0 = gs[2 * i], g1 = gs[2 * i + 1];
        v0 = make_float4(v0.x * g0.x, v0.y * g0.y, v0.z * g0.z, v0.w * g0.w);
        v1 = make_float4(v1.x * g1.x, v1.y * g1.y, v1.z * g1.z, v1.w * g1.w);
      }
      if (P.need_f32) {
        reinterpret_cast<float4*>(xf)[2 * i] = v0;
        reinterpret_cast<float4*>(xf)[2 * i + 1] = v1;
      }
    }
    quantize_item(v0, v1, i, in, U, lim, ucon);
  }
  if (norm) {
    ss = warp_sum(ss);
    if (lane == 0) dred[warp] = ss;
  }
  consumer_sync(NC);  // limbs, unit constants, sums of squares (and the fp32 copy) are visible
  return true;
}

template <uint32_t TM>
__global__ void __launch_bounds__(kMaxThreads, 1) gemv_kernel(const __grid_constant__ GemvArgs A,
                                                              const __grid_constant__ Plan P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = A.K, U = P.U, S = P.S, NS = P.stages, NC = P.NC;
  const int Ur = U | 1;  // row stride of the partial sums
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // ---- shared-memory carve-up (must match fixed_bytes())
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);              // [kMaxStages]
  uint64_t* empty = full + kMaxStages;                             // [kMaxStages]
  uint64_t* xready = reinterpret_cast<uint64_t*>(smem + 512);      // x staged (one arrival)
  StageDesc* desc = reinterpret_cast<StageDesc*>(smem + 128);      // [kMaxStages]
  double* dred = reinterpret_cast<double*>(smem + 384);            // [16]
  float* ucon = reinterpret_cast<float*>(smem + 640);              // g[U], ga[4][U]
  uint4* lim = reinterpret_cast<uint4*>(smem + 640 + ((20 * U + 127) & ~127));  // [12][U]
  float* red = reinterpret_cast<float*>(lim + 12 * U);             // [2][red_floats] (x, gains first)
  float* xf = reinterpret_cast<float*>(                            // [K] (F32 weights only)
      (reinterpret_cast<uintptr_t>(red + 2 * P.red_floats) + 15) & ~uintptr_t(15));
  const uintptr_t sp = reinterpret_cast<uintptr_t>(xf + (P.need_f32 ? K : 0));
  uint8_t* stages = reinterpret_cast<uint8_t*>((sp + 127) & ~uintptr_t(127));

  const int n_stages = count_stages(P);
  if (n_stages == 0) return;  // no rows for this CTA
  if (tid == NC) {  // producer lane: barriers
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NC / 32);
    }
    mbar_init(xready, 1);
    fence_barrier_init();
  }
  __syncthreads();

  if (tid >= NC) {
    // ============================================================ producer
    if (tid != NC) return;
    // the first stages go out before the grid-dependency wait
    Cursor cur;
    cur.ls = 0;
    cta_rows(P, 0, &cur.r, &cur.hi);
    cursor_seek(P, &cur);
    const uint64_t pol = policy_evict_first();
    const int first = NS < n_stages ? NS : n_stages, pre = kPreStages < first ? kPreStages : first;
    for (int i = 0; i < pre; ++i)
      issue_next(A, P, &cur, stages + (size_t)i * P.stage_bytes, &desc[i], &full[i], pol);
    grid_dep_wait();  // *active is written by the previous kernel
    grid_dep_launch();
    if (A.active && __ldcg(A.active) == 0) {  // drain the copies in flight, then leave
      for (int i = 0; i < pre; ++i) mbar_wait(&full[i], 0, A.err);
      return;
    }
    if (kXGate && pre < first) mbar_wait(xready, 0, A.err);
    for (int i = pre; i < first; ++i)
      issue_next(A, P, &cur, stages + (size_t)i * P.stage_bytes, &desc[i], &full[i], pol);
    for (int it = NS; it < n_stages; ++it) {
      const int slot = it % NS;
      mbar_wait(&empty[slot], (uint32_t)(it / NS - 1) & 1u, A.err);
      issue_next(A, P, &cur, stages + (size_t)slot * P.stage_bytes, &desc[slot], &full[slot], pol);
    }
    prefetch_next(A);
    return;
  }

  // ============================================================== consumers
  if (!prologue(A, P, tid, lane, warp, dred, lim, ucon, xf, reinterpret_cast<float4*>(red), xready)) return;
  float nscale = 1.0f;
  if (A.norm_w) {  // RMSNorm factor of x (sum of squares in double, fixed order)
    double tot = 0.0;
#pragma unroll 1
    for (int w = 0; w < NC / 32; ++w) tot += dred[w];
    nscale = 1.0f / sqrtf((float)tot / (float)K + A.eps);
  }

  const int u = tid % U, s = tid / U;
  const bool busy = s < S;
  const UnitOff uo = unit_offsets(u);
  const uint32_t stages32 = smem_u32(stages);
  ActR act;
  if (busy) {
#pragma unroll
    for (int L = 0; L < 3; ++L) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = lim[(L * 4 + j) * U + u];
        act.a[L][4 * j] = v.x;
        act.a[L][4 * j + 1] = v.y;
        act.a[L][4 * j + 2] = v.z;
        act.a[L][4 * j + 3] = v.w;
      }
    }
    act.g = ucon[u];
#pragma unroll
    for (int j = 0; j < 4; ++j) act.ga[j] = ucon[(1 + j) * U + u];
  }

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
    const uint32_t sb = stages32 + (uint32_t)slot * (uint32_t)P.stage_bytes;
    if (busy) {
      // pairs: gate and up row j; otherwise rows j and j + S (row j twice
      // when j + S is past the stage, the second result dropped)
      const uint32_t base0 = sb + d.off0;
      const uint32_t base1 = L.pair ? sb + d.off1 : base0;
      const int step = L.pair ? S : 2 * S, second = L.pair ? 0 : S;
#pragma unroll 1
      for (int j = s; j < d.n; j += step) {
        const int j2 = j + second;
        const bool has2 = L.pair || j2 < d.n;
        const uint32_t ba[2] = {base0 + (uint32_t)(j * rb), base1 + (uint32_t)((has2 ? j2 : j) * rb)};
        float y[2];
        unit_rows<2, TM>(type, ba, u, uo, act, xf, y);
        rbuf[(jr0 + j) * Ur + u] = y[0];
        if (L.pair) rbuf[(ck_rows + jr0 + j) * Ur + u] = y[1];
        else if (has2) rbuf[(jr0 + j2) * Ur + u] = y[1];
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
    consumer_sync(NC);
    const int rows = jr0 + d.n;
    const int nsum = rows * (L.pair + 1);
#pragma unroll 1
    for (int b0 = 0; b0 < 4 * nsum; b0 += NC) {  // warp-uniform trip count
      const int idx = b0 + tid, q = idx & 3, sid = idx >> 2;
      const int j = L.pair ? sid >> 1 : sid, h = L.pair ? sid & 1 : 0;
      float t = 0.0f;
      if (sid < nsum) {
        const float* p = rbuf + (h * ck_rows + j) * Ur;
#pragma unroll 4
        for (int v = q; v < U; v += 4) t += p[v];
      }
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      t *= nscale;
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
  if (a.nseg < 1 || a.nseg > 4 || a.K <= 0 || a.K % 128 != 0) return false;
  const int U = a.K / 64;
  if (U > kMaxConsumers) return false;
  P->U = U;
  P->S = kMaxConsumers / U;
  P->NC = (U * P->S + 31) & ~31;

  if (a.npf < 0 || a.npf > 4 || a.pf_bytes < 0) return false;
  for (int i = 0; i < a.npf; ++i)  // 32-bit row arithmetic in the prefetch
    if (a.pf[i].rows < 0 || a.pf[i].rows > (int64_t)(0xFFFFFFFFu / 1024) || a.pf[i].row_bytes < 0 ||
        a.pf[i].rows * a.pf[i].row_bytes > (int64_t)0xFFFFFFFFu)
      return false;
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
    // a round gives every slot two rows (a gate/up pair, or rows j and j + S)
    const int64_t per_round = (int64_t)P->S * G.row_bytes * 2;
    int64_t rounds = kStageTarget / per_round;
    if (rounds < 1) rounds = 1;
    L.m = (int32_t)(rounds * P->S * (L.pair ? 1 : 2));
    const int64_t slot = ((int64_t)L.m * G.row_bytes + 32 + 127) & ~int64_t(127);
    if (slot > kSmemLimit / 3) return false;
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
  // the partial-sum buffers first hold x (and the gains) during the prologue
  const int stage_floats = a.K * (a.norm_w ? 2 : 1);
  if (2 * red < stage_floats) red = (stage_floats + 1) / 2;
  P->stage_bytes = stage_bytes;
  P->half_bytes = half_bytes;
  P->red_floats = red;
  return true;
}

size_t fixed_bytes(const Plan& P, int K) {
  const size_t b = 640 + (((size_t)20 * P.U + 127) & ~size_t(127)) + (size_t)12 * 16 * P.U +
                   (((size_t)2 * P.red_floats * 4 + 15) & ~size_t(15)) + (P.need_f32 ? (size_t)K * 4 : 0);
  return (b + 127) & ~size_t(127);
}

// Kernel instantiations by type mix.
template <uint32_t TM>
void configure(int dev) {
  static bool done[64] = {false};
  if (dev < 0 || dev >= 64 || done[dev]) return;
  cudaFuncSetAttribute(gemv_kernel<TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
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

bool gemv_supported(int64_t K, bool norm) {
  (void)norm;
  return K > 0 && K % 128 == 0 && K / 64 <= kMaxConsumers;
}

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
  cfg.blockDim = dim3(P.NC + 32);
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
