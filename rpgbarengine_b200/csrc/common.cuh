// common.cuh -- device helpers shared by the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define RPGC_DEV __device__ __forceinline__

namespace rpgc {

constexpr uint32_t kF32 = 0, kF16 = 1, kQ8_0 = 8, kQ4_K = 12, kQ6_K = 14;

// Error flag bits written by kernels whose bounded waits gave up.
constexpr int kErrTimeout = 1;

// Upper bound of polls of one mbarrier phase before a wait gives up
// (each poll already blocks for a hardware-chosen interval).
constexpr uint32_t kMaxPolls = 1u << 20;

// ------------------------------------------------------------- halves
// Exact IEEE binary16 -> binary32 by bit manipulation, subnormals
// normalised by hand, Inf/NaN payload carried (reference src/dtypes.h:21-47).
RPGC_DEV float f16_bits_to_f32(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t out;
  if (exp == 0) {
    if (man == 0) {
      out = sign;
    } else {
      const int s = __clz(man) - 21;  // shifts that bring bit 10 to the top
      man = (man << s) & 0x3FFu;
      out = sign | ((uint32_t)(113 - s) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    out = sign | 0x7F800000u | (man << 13);
  } else {
    out = sign | ((exp + 112u) << 23) | (man << 13);
  }
  return __uint_as_float(out);
}

RPGC_DEV uint32_t ld_u16(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
}

// Q4_K / Q5_K 6-bit (scale, min) unpack of sub-block j (ggml get_scale_min_k4).
RPGC_DEV void scale_min_k4(int j, const uint8_t* q, uint32_t* sc, uint32_t* m) {
  if (j < 4) {
    *sc = q[j] & 63u;
    *m = q[j + 4] & 63u;
  } else {
    *sc = (q[j + 4] & 0x0Fu) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// One dequantised element e of a row, bit-exact with the reference's
// DequantizeRow (src/quant.cc:207-217, 327-354, 396-429): the separate
// roundings of the reference are kept with __fmul_rn/__fsub_rn so that no
// multiply-add is contracted.
RPGC_DEV float deq_elem(uint32_t type, const uint8_t* row, int64_t e) {
  if (type == kF32) return __ldg(reinterpret_cast<const float*>(row) + e);
  if (type == kF16) return f16_bits_to_f32(ld_u16(row + 2 * e));
  if (type == kQ8_0) {
    const uint8_t* p = row + (e >> 5) * 34;
    const float d = f16_bits_to_f32(ld_u16(p));
    return __fmul_rn((float)(int8_t)p[2 + (e & 31)], d);
  }
  if (type == kQ4_K) {
    const uint8_t* p = row + (e >> 8) * 144;
    const int i = (int)(e & 255), g = i >> 6, hi = (i >> 5) & 1, l = i & 31;
    uint32_t sc, m;
    scale_min_k4(2 * g + hi, p + 4, &sc, &m);
    const float d = f16_bits_to_f32(ld_u16(p)), dmin = f16_bits_to_f32(ld_u16(p + 2));
    const uint8_t b = p[16 + 32 * g + l];
    const uint32_t q = hi ? (b >> 4) : (b & 15u);
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
  }
  // kQ6_K
  const uint8_t* p = row + (e >> 8) * 210;
  const int i = (int)(e & 255), h = i >> 7, r = i & 127, qd = r >> 5, l = r & 31;
  const uint8_t lb = p[64 * h + l + 32 * (qd & 1)];
  const uint32_t nib = (qd >= 2) ? (lb >> 4) : (lb & 15u);
  const uint32_t hb = (p[128 + 32 * h + l] >> (2 * qd)) & 3u;
  const int q = (int)(nib | (hb << 4)) - 32;
  const int sc = (int8_t)p[192 + 8 * h + (l >> 4) + 2 * qd];
  const float d = f16_bits_to_f32(ld_u16(p + 208));
  return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

// ------------------------------------------------------------ dp4a
// Byte-wise dot products with int32 accumulation.  Weights are the first
// operand (u8 for K-quants, s8 for Q8_0), activation limbs the second.
RPGC_DEV int dp4a_us(uint32_t a, uint32_t b, int c) {  // a unsigned, b signed
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
RPGC_DEV int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
RPGC_DEV int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
RPGC_DEV int dp4a_su(uint32_t a, uint32_t b, int c) {  // a signed, b unsigned
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ------------------------------------------------------ reductions
template <typename T>
RPGC_DEV T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
RPGC_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------ mbarrier / bulk copy
RPGC_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
RPGC_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
RPGC_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
RPGC_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
RPGC_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
RPGC_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that may suspend the thread up to `ns` nanoseconds (woken early
// when the phase completes), so a waiting warp does not spin on the issue
// slots other warps need.
RPGC_DEV bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Bounded wait with suspension: at most kMaxSleepPolls polls of up to 2 us.
constexpr uint32_t kMaxSleepPolls = 1u << 19;
RPGC_DEV bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kMaxSleepPolls; ++i)
    if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
  if (err) atomicOr(err, kErrTimeout);
  return false;
}
// Bounded wait: returns false (and sets the error flag) if the phase never
// completed within kMaxPolls polls.
RPGC_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kMaxPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, kErrTimeout);
  return false;
}
// Bulk global -> shared copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completion counted on `bar`.  Streaming data: evict-first.
RPGC_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                       uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
RPGC_DEV uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Programmatic dependent launch: wait for the producer grid's memory.
RPGC_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
RPGC_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// Launch with programmatic stream serialisation: the kernel may be scheduled
// while the previous kernel in the stream finishes, and must execute
// grid_dep_wait() before it touches memory that kernel reads or writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// Unaligned little-endian 32-bit word from shared memory built from the two
// aligned words around it.
RPGC_DEV uint32_t lds_u32(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  return sh ? __funnelshift_r(w[0], w[1], sh) : w[0];
}

// n consecutive unaligned words starting at p (n+1 aligned loads).
template <int N>
RPGC_DEV void lds_words(const uint8_t* p, uint32_t* out) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  if (sh == 0) {
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = w[j];
  } else {
    uint32_t prev = w[0];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const uint32_t nx = w[j + 1];
      out[j] = __funnelshift_r(prev, nx, sh);
      prev = nx;
    }
  }
}

}  // namespace rpgc
