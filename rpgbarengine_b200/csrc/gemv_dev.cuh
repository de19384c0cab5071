// gemv_dev.cuh -- device building blocks of the decode matrix-vector
// product shared by the per-launch GEMV (k_gemv.cu) and the persistent
// decode-step kernel (k_step.cu): the activation unit in registers, the
// per-format unit products on 32-bit shared addresses, and the cooperative
// fixed-point quantisation of the activation.  See k_gemv.cu for the work
// split and the arithmetic.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace rpgc {
namespace gemv {

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

// Position in a ring of NS slots: the slot and the parity of its current use
// (kept incrementally: no division per stage).
struct RingPos {
  int slot = 0;
  uint32_t parity = 0;
  bool wrapped = false;  // every slot has been used once
  __device__ __forceinline__ void advance(int ns) {
    if (++slot == ns) {
      slot = 0;
      parity ^= 1u;
      wrapped = true;
    }
  }
};

// One thread's rows of a stage of n rows: rows j = s, s + step, ... (pairs:
// gate row j and up row j; otherwise rows j and j + S, row j twice when
// j + S is past the stage and the second result dropped).  The partial of
// row j goes to p0[j * Ur + u] (up row: p1[j * Ur + u]).  The block format is
// fixed for the loop.
template <int KIND>
__device__ __forceinline__ void rows_of_stage(uint32_t base0, uint32_t base1, int n, int s, int S, bool pair,
                                              int rb, int u, int Ur, const UnitOff& uo, const ActR& act,
                                              const float* xf, float* p0, float* p1) {
  const int step = pair ? S : 2 * S, second = pair ? 0 : S;
#pragma unroll 1
  for (int j = s; j < n; j += step) {
    const int j2 = j + second;
    const bool has2 = pair || j2 < n;
    const uint32_t ba[2] = {base0 + (uint32_t)(j * rb), base1 + (uint32_t)((has2 ? j2 : j) * rb)};
    float y[2];
    if constexpr (KIND == 0) q4k_unit<2>(ba, uo, act, y);
    else if constexpr (KIND == 1) q6k_unit<2>(ba, uo, act, y);
    else if constexpr (KIND == 2) q8_0_unit<2>(ba, uo, act, y);
    else f32_unit<2>(ba, u, xf, y);
    p0[j * Ur + u] = y[0];
    if (pair) p1[j * Ur + u] = y[1];
    else if (has2) p0[j2 * Ur + u] = y[1];
  }
}

template <uint32_t TM>
__device__ __forceinline__ void stage_rows(uint32_t type, uint32_t base0, uint32_t base1, int n, int s, int S,
                                           bool pair, int rb, int u, int Ur, const UnitOff& uo, const ActR& act,
                                           const float* xf, float* p0, float* p1) {
  if ((TM & kMQ4K) && type == kQ4_K)
    rows_of_stage<0>(base0, base1, n, s, S, pair, rb, u, Ur, uo, act, xf, p0, p1);
  else if ((TM & kMQ6K) && type == kQ6_K)
    rows_of_stage<1>(base0, base1, n, s, S, pair, rb, u, Ur, uo, act, xf, p0, p1);
  else if ((TM & kMQ80) && type == kQ8_0)
    rows_of_stage<2>(base0, base1, n, s, S, pair, rb, u, Ur, uo, act, xf, p0, p1);
  else if (TM & kMF32)
    rows_of_stage<3>(base0, base1, n, s, S, pair, rb, u, Ur, uo, act, xf, p0, p1);
}

// 16-byte asynchronous global -> shared copy through L2 (not L1: the source
// may have been written by the previous kernel).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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

}  // namespace gemv
}  // namespace rpgc
