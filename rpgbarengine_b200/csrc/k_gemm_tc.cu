// k_gemm_tc.cu -- prefill matmul over raw ggml blocks on the 5th-generation
// tensor cores (tcgen05, sm_100a).
//
// Replaces the reference's blocked multi-token kernel (MatMulBlocked,
// src/matmul_avx2.cc:482-507, called by QuantMatrix::MatMulBatch,
// src/model.cc:32-69): OUT[t][r] (+)= dot(X[t], W[r]).
//
// Precision.  The tensor cores multiply fp16 operands into fp32.  Each
// weight is dequantised to the reference's fp32 value (Q4_K: within one
// rounding of it) and split into fp16 hi + lo (W = Wh + Wl to 2^-22); each
// token row of X is scaled by
// a power of two and split the same way (X s = Xh + Xl).  Three products
// Xh Wh + Xh Wl + Xl Wh accumulate over the whole K in TMEM; the dropped
// Xl Wl term and the fp16 roundings leave ~2^-21 of sum|a w|, inside the
// per-row gate 1e-5.  The epilogue divides by the token's scale.
//
// Data path (one CTA per 256 tokens x 128 weight rows):
//   warp 0      TMA of the Xh / Xl tiles (SWIZZLE_128B, 64 K x 256 tokens)
//   warp 1      TMEM allocation and the MMA issue (one thread): per 64-K
//               stage 2 token blocks (1 when the tile's second 128 tokens
//               are past n, e.g. a batched decode step) x 4 k16 steps x 3
//               products, M=128 N=128 K=16 each, then tcgen05.commit frees
//               the stage
//   warps 2..   dequantise the stage's weight tile into Wh / Wl (same
//               swizzled K-major layout; four threads per row), then read
//               the two 128 x TN fp32 accumulators back from TMEM and
//               write OUT
// Two 96 KB stages; all waits are bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_dev.cuh"

namespace rpgc {
namespace {

using namespace tc;

constexpr int TMt = 256;  // tokens per CTA
constexpr int TKt = 64;   // K per stage (one 128-byte swizzle row of fp16)
constexpr int kStg = 2;
constexpr int kABytes = TMt * TKt * 2;   // one of Xh / Xl per stage

// Geometry of a tile of TN weight rows (TN = 96, 128 or 144: the launcher
// takes the one with the least work per SM).  Four dequant threads per row,
// 16 weights each per stage.
template <int TN>
struct Tile {
  static constexpr int kDeqWarps = TN / 8;
  static constexpr int kThreads = (2 + kDeqWarps) * 32;
  static constexpr int kWBytes = TN * TKt * 2;  // one of Wh / Wl per stage
  static constexpr int kStageBytes = 2 * kABytes + 2 * kWBytes;
  static constexpr int kSmem = kStg * kStageBytes + 1024 + 1024;  // + barriers, + alignment slack
  static constexpr uint32_t kTmemCols = 2 * TN <= 256 ? 256u : 512u;  // two 128 x TN accumulators
  // instruction descriptor: fp16 x fp16 -> fp32, both K-major, M = 128, N = TN
  static constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
  static_assert(TN % 16 == 0 && TN <= 256 && kSmem <= 227 * 1024, "tile");
};

// One matrix of a launch: blockIdx.x counts the tiles of the matrices in order
// (a group of matrices with the same input, e.g. q, k and v, is one launch).
struct GemmMat {
  const uint8_t* w;
  int64_t rows, row_bytes;
  float* out;             // ks == 1: OUT; else the partial sums [ks][n][rows]
  int64_t ldo;
  uint32_t type;
  int32_t tiles;          // row tiles of this matrix
};

struct GemmArgs {
  GemmMat mat[3];
  int32_t nmat;
  int64_t K;
  int64_t n;              // tokens
  int32_t ks;             // K partitions (gridDim.z; 1 for a group)
  const float* inv_scale; // per token
  int32_t* err;
  int32_t accumulate;
  const float* glu;       // ks == 1, optional: OUT = silu(glu) * (X W^T), glu in OUT's layout
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------ dequant
// Aligned little-endian words covering an arbitrary 2-byte-aligned global
// range, realigned by funnel shifts: N words starting at p.
template <int N>
__device__ __forceinline__ void ldg_words(const uint8_t* p, uint32_t* out) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  uint32_t prev = __ldg(w);
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t nx = __ldg(w + j + 1);
    out[j] = __funnelshift_r(prev, nx, sh);
    prev = nx;
  }
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w0, uint32_t w1, uint32_t w2, int k) {
  const uint32_t w = k < 4 ? w0 : (k < 8 ? w1 : w2);
  return (w >> (8 * (k & 3))) & 0xFFu;
}

// Raw bytes of 16 weights [k0, k0 + 16) of one row (k0 a multiple of 16),
// fetched two stages ahead of their use so that the global-memory latency
// hides behind the dequantisation of the stages in between.
constexpr int kRaw = 10;  // words
__device__ __forceinline__ void fetch16(uint32_t type, const uint8_t* row, int64_t k0, uint32_t* r) {
  if (type == kQ4_K) {  // header + 16 quant bytes (both nibble planes)
    const uint8_t* blk = row + (k0 >> 8) * 144;
    const int i0 = (int)(k0 & 255);
    const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(blk));
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * (i0 >> 6) + (i0 & 31)));
    r[0] = hdr.x; r[1] = hdr.y; r[2] = hdr.z; r[3] = hdr.w;
    r[4] = q.x; r[5] = q.y; r[6] = q.z; r[7] = q.w;
  } else if (type == kQ6_K) {  // 16 ql bytes, 16 qh bytes, the scale pair, d
    const uint8_t* blk = row + (k0 >> 8) * 210;
    const int i0 = (int)(k0 & 255), h = i0 >> 7, qd = (i0 & 127) >> 5, o = i0 & 16;
    ldg_words<4>(blk + 64 * h + 32 * (qd & 1) + o, r);
    ldg_words<4>(blk + 128 + 32 * h + o, r + 4);
    ldg_words<1>(blk + 192 + 8 * h + 2 * qd, r + 8);
    ldg_words<1>(blk + 208, r + 9);
  } else if (type == kQ8_0) {  // d, then the 16 quants from a word boundary
    const uint8_t* blk = row + (k0 >> 5) * 34;
    ldg_words<1>(blk, r);
    ldg_words<4>(blk + 2 + (k0 & 16), r + 1);
  }
}

// Byte J of w as a float without the conversion unit: the float with bits
// 0x4B000000 | byte is 2^23 + byte; `bias` removes 2^23 and any offset of
// the format (exact: every operand is an integer below 2^24).
template <int J>
__device__ __forceinline__ float byte_as_f(uint32_t w, float bias) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + J)) - bias;
}

// kWScale * the 32 weights from their raw bytes: the reference's
// DequantizeRow values (src/quant.cc:207-217, 327-354, 396-429) on scales
// premultiplied by the power of two kWScale (which commutes with every
// rounding; it keeps the fp16 lo halves of the split out of the subnormal
// range).  Q6_K and Q8_0 take the reference's single product, so they are
// its values exactly; Q4_K's d*sc*q - dmin*m is one fused multiply-add, at
// most one rounding (2^-24 relative) from the reference's two, far below the
// split's 2^-22.  F32 rows are read here.
constexpr float kWScale = 256.0f;
__device__ __forceinline__ void convert16(uint32_t type, const uint32_t* r, const uint8_t* row,
                                          int64_t k0, float* w) {
  if (type == kQ4_K) {
    const int i0 = (int)(k0 & 255), g = i0 >> 6, half = (i0 >> 5) & 1, j = 2 * g + half;
    uint32_t sc, m;
    if (j < 4) {
      sc = byte_of(r[1], r[2], r[3], j) & 63u;
      m = byte_of(r[1], r[2], r[3], j + 4) & 63u;
    } else {
      sc = (byte_of(r[1], r[2], r[3], j + 4) & 0x0Fu) | ((byte_of(r[1], r[2], r[3], j - 4) >> 6) << 4);
      m = (byte_of(r[1], r[2], r[3], j + 4) >> 4) | ((byte_of(r[1], r[2], r[3], j) >> 6) << 4);
    }
    const float d = f16_bits_to_f32(r[0] & 0xFFFFu), dmin = f16_bits_to_f32(r[0] >> 16);
    const float ds = __fmul_rn(d, (float)sc) * kWScale, ndm = -(__fmul_rn(dmin, (float)m) * kWScale);
    const uint32_t sh = 4u * (uint32_t)half;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t nb = (r[4 + i] >> sh) & 0x0F0F0F0Fu;  // four quants, one per byte
      w[4 * i] = fmaf(ds, byte_as_f<0>(nb, 8388608.0f), ndm);
      w[4 * i + 1] = fmaf(ds, byte_as_f<1>(nb, 8388608.0f), ndm);
      w[4 * i + 2] = fmaf(ds, byte_as_f<2>(nb, 8388608.0f), ndm);
      w[4 * i + 3] = fmaf(ds, byte_as_f<3>(nb, 8388608.0f), ndm);
    }
  } else if (type == kQ6_K) {
    const int i0 = (int)(k0 & 255), qd = (i0 & 127) >> 5;
    const float d = f16_bits_to_f32(r[9] & 0xFFFFu);
    const uint32_t scb = (i0 & 16) ? (r[8] >> 8) & 0xFFu : r[8] & 0xFFu;  // 16 weights share one scale
    const float dsc = __fmul_rn(d, (float)(int)(int8_t)scb) * kWScale;
    const uint32_t nsh = qd >= 2 ? 4u : 0u, hsh = 2u * (uint32_t)qd;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // q + 32 = low 4 bits from ql, high 2 from qh, four per word
      const uint32_t q = ((r[i] >> nsh) & 0x0F0F0F0Fu) | (((r[4 + i] >> hsh) & 0x03030303u) << 4);
      w[4 * i] = __fmul_rn(dsc, byte_as_f<0>(q, 8388640.0f));  // 2^23 + 32
      w[4 * i + 1] = __fmul_rn(dsc, byte_as_f<1>(q, 8388640.0f));
      w[4 * i + 2] = __fmul_rn(dsc, byte_as_f<2>(q, 8388640.0f));
      w[4 * i + 3] = __fmul_rn(dsc, byte_as_f<3>(q, 8388640.0f));
    }
  } else if (type == kQ8_0) {
    const float d = f16_bits_to_f32(r[0] & 0xFFFFu) * kWScale;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t f = r[1 + i] ^ 0x80808080u;  // quants with the sign bit flipped: q + 128
      w[4 * i] = __fmul_rn(byte_as_f<0>(f, 8388736.0f), d);  // 2^23 + 128
      w[4 * i + 1] = __fmul_rn(byte_as_f<1>(f, 8388736.0f), d);
      w[4 * i + 2] = __fmul_rn(byte_as_f<2>(f, 8388736.0f), d);
      w[4 * i + 3] = __fmul_rn(byte_as_f<3>(f, 8388736.0f), d);
    }
  } else {  // F32
    const float4* p = reinterpret_cast<const float4*>(row + k0 * 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = __ldg(p + i);
      w[4 * i] = v.x * kWScale;
      w[4 * i + 1] = v.y * kWScale;
      w[4 * i + 2] = v.z * kWScale;
      w[4 * i + 3] = v.w * kWScale;
    }
  }
}

template <int TN>
__global__ void __launch_bounds__(Tile<TN>::kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_h,
                                                                        const __grid_constant__ CUtensorMap tm_l,
                                                                        const GemmArgs g) {
  using T = Tile<TN>;
  constexpr int kStageBytes = T::kStageBytes, kWBytes = T::kWBytes, kDeqWarps = T::kDeqWarps;
  constexpr uint32_t kTmemCols = T::kTmemCols;
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* gsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(gsm + kStg * kStageBytes);
  uint64_t* full_a = bars;              // [kStg] TMA bytes of the X tiles
  uint64_t* full_w = bars + kStg;       // [kStg] the dequant warps
  uint64_t* empty = bars + 2 * kStg;    // [kStg] MMAs of the stage done
  uint64_t* acc_full = bars + 3 * kStg; // all MMAs done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * kStg + 1);
  auto Ah = [&](int s) { return gsm + s * kStageBytes; };
  auto Al = [&](int s) { return gsm + s * kStageBytes + kABytes; };
  auto Wh = [&](int s) { return gsm + s * kStageBytes + 2 * kABytes; };
  auto Wl = [&](int s) { return gsm + s * kStageBytes + 2 * kABytes + kWBytes; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int bx = (int)blockIdx.x, mi = 0;  // the matrix of this CTA and its tile there
  while (mi + 1 < g.nmat && bx >= g.mat[mi].tiles) bx -= g.mat[mi++].tiles;
  const GemmMat& M = g.mat[mi];
  const int64_t n0 = (int64_t)bx * TN;           // first weight row
  const int t0 = (int)blockIdx.y * TMt;          // first token
  const int nk_all = (int)(g.K / TKt);
  const int nmb = g.n - t0 > 128 ? 2 : 1;        // 128-token halves holding live tokens
  const int kc0 = (int)((int64_t)nk_all * blockIdx.z / g.ks);  // this CTA's stages
  const int nk = (int)((int64_t)nk_all * (blockIdx.z + 1) / g.ks) - kc0;
  // Launched as a programmatic dependent: the set-up, the TMEM allocation and
  // the weight stages (which no kernel writes) overlap the previous kernel's
  // tail; X (warp 0) and the epilogue's reads and writes wait for it.  The
  // next kernel may start its own set-up as soon as every CTA here has begun.
  grid_dep_launch();

  if (tid == 0) {
    for (int s = 0; s < kStg; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&full_w[s], kDeqWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (X tiles)
    if (lane == 0) {
      grid_dep_wait();  // X is the previous kernel's output
      for (int c = 0; c < nk; ++c) {
        const int s = c % kStg;
        if (c >= kStg) mbar_wait_sleep(&empty[s], (uint32_t)(c / kStg - 1) & 1u, g.err);
        mbar_arrive_expect_tx(&full_a[s], 2 * kABytes);
        tma_load_2d(Ah(s), &tm_h, (kc0 + c) * TKt, t0, &full_a[s]);
        tma_load_2d(Al(s), &tm_l, (kc0 + c) * TKt, t0, &full_a[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issue
    if (lane == 0) {
      for (int c = 0; c < nk; ++c) {
        const int s = c % kStg;
        const uint32_t ph = (uint32_t)(c / kStg) & 1u;
        mbar_wait_sleep(&full_a[s], ph, g.err);
        mbar_wait_sleep(&full_w[s], ph, g.err);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < TKt / 16; ++kk) {
          const uint64_t bh = sdesc(Wh(s) + kk * 32), bl = sdesc(Wl(s) + kk * 32);
#pragma unroll
          for (int mb = 0; mb < 2; ++mb) {
            if (mb >= nmb) break;  // a half past the last token: no MMAs for it
            const uint64_t ah = sdesc(Ah(s) + mb * (128 * 128) + kk * 32);
            const uint64_t al = sdesc(Al(s) + mb * (128 * 128) + kk * 32);
            const uint32_t d = tmem + (uint32_t)(mb * TN);
            mma_f16(d, ah, bh, T::kIdesc, (c > 0 || kk > 0) ? 1u : 0u);
            mma_f16(d, ah, bl, T::kIdesc, 1u);
            mma_f16(d, al, bh, T::kIdesc, 1u);
          }
        }
        mma_commit(&empty[s]);  // the stage may be refilled once these MMAs are done
      }
      mma_commit(acc_full);
    }
  } else {
    // ------------------------------------------------ weight dequant
    const int dt = tid - 64;                 // 0 .. 4 TN - 1
    const int r = dt >> 2, qq = dt & 3;      // tile row, 16-element quarter of the stage's 64
    const int64_t gr = n0 + r;
    const uint8_t* row = M.w + gr * M.row_bytes;
    // Raw bytes run two stages ahead: the loads for stage c + 2 are issued
    // after stage c is published (the proxy fence would otherwise wait for
    // them), and consumed after stage c + 1 has been processed.
    const bool live = gr < M.rows;
    uint32_t raw0[kRaw], raw1[kRaw];
    if (live) {
      fetch16(M.type, row, (int64_t)kc0 * TKt + 16 * qq, raw0);
      if (nk > 1) fetch16(M.type, row, (int64_t)(kc0 + 1) * TKt + 16 * qq, raw1);
    }
    // stage c converts the raw words fetched two stages earlier, then fetches
    // stage c + 2 into the same registers (even stages raw0, odd raw1: the
    // loop runs two stages per pass so that no register copy waits on a load)
    auto stage = [&](int c, uint32_t* raw) {
      const int s = c % kStg;
      const int64_t k0 = (int64_t)(kc0 + c) * TKt + 16 * qq;
      float w[16];
      if (live) {
        convert16(M.type, raw, row, k0, w);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = 0.0f;
      }
      if (c >= kStg) mbar_wait_sleep(&empty[s], (uint32_t)(c / kStg - 1) & 1u, g.err);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint4 hi, lo;
        split8(w + 8 * q, &hi, &lo);
        const uint32_t off = swz(r, 2 * qq + q);
        *reinterpret_cast<uint4*>(Wh(s) + off) = hi;
        *reinterpret_cast<uint4*>(Wl(s) + off) = lo;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the MMA
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_w[s]);
      if (live && c + 2 < nk) fetch16(M.type, row, k0 + 2 * TKt, raw);
    };
    static_assert(kStg == 2, "the raw words alternate between two register sets");
    for (int c = 0; c < nk; c += 2) {
      stage(c, raw0);
      if (c + 1 < nk) stage(c + 1, raw1);
    }
    // ------------------------------------------------ epilogue
    // the dequant warps read the accumulators: warp w may read TMEM lanes
    // 32 (w % 4) .. + 31 only, so the nq warps with one w % 4 share that
    // quarter of both token halves mb (the first eight warps take one
    // (half, quarter) each, the others none)
    grid_dep_wait();  // OUT, the partial sums, glu and the row scales belong to earlier kernels
    mbar_wait_sleep(acc_full, 0, g.err);
    tc_fence_after();
    const int ew = warp - 2, quarter = warp & 3, nq = (kDeqWarps - (ew & 3) + 3) >> 2;
#pragma unroll 1
    for (int mb = ew >> 2; mb < nmb; mb += nq) {
      const int tl = mb * 128 + quarter * 32 + lane;  // token row of the tile = TMEM lane
      const int64_t t = t0 + tl;
      const float inv = t < g.n ? g.inv_scale[t] : 0.0f;
      const bool part = g.ks > 1;
      float* obase = part ? M.out + ((int64_t)blockIdx.z * g.n + t) * M.rows : M.out + t * M.ldo;
      const float* gbase = g.glu ? g.glu + t * M.ldo : nullptr;
      // 16-byte accesses when the token's rows are 16-byte aligned (n0 and the
      // 16-column runs keep that alignment)
      const bool vec = ((reinterpret_cast<uintptr_t>(obase) | reinterpret_cast<uintptr_t>(gbase)) & 15) == 0;
#pragma unroll 1
      for (int j = 0; j < TN / 16; ++j) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(mb * TN + 16 * j), v);
        if (t < g.n) {
          float* o = obase + n0 + 16 * j;
          const int64_t lim = M.rows - (n0 + 16 * j);  // columns left in the matrix
          if (lim >= 16 && vec) {  // whole 64-byte run of the token's row: 16-byte accesses
            const float* gp = gbase ? gbase + n0 + 16 * j : nullptr;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float4 y = make_float4(v[4 * q] * inv, v[4 * q + 1] * inv, v[4 * q + 2] * inv, v[4 * q + 3] * inv);
              float4* op = reinterpret_cast<float4*>(o) + q;
              if (gp) {
                const float4 gv = reinterpret_cast<const float4*>(gp)[q];
                y.x *= gv.x / (1.0f + expf(-gv.x));
                y.y *= gv.y / (1.0f + expf(-gv.y));
                y.z *= gv.z / (1.0f + expf(-gv.z));
                y.w *= gv.w / (1.0f + expf(-gv.w));
              } else if (g.accumulate && !part) {
                const float4 p = *op;
                y.x += p.x;
                y.y += p.y;
                y.z += p.z;
                y.w += p.w;
              }
              *op = y;
            }
            continue;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (i < lim) {
              const float y = v[i] * inv;
              if (gbase) {  // SwiGLU with the gate projection already in OUT's layout
                const float gv = gbase[n0 + 16 * j + i];
                o[i] = (gv / (1.0f + expf(-gv))) * y;
              } else {
                o[i] = (g.accumulate && !part) ? o[i] + y : y;
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

// Per token row: the values v (mode kPlain: x; kNorm: the RMSNorm of x,
// src/kernels.h:56-63, x * (1/sqrt(sum x^2 / K + eps), double sum) * w;
// kGlu: silu(gate) * up, src/kernels.h:82-92, as swiglu_kernel), a
// power-of-two scale s (max |v| s in [2^14, 2^15)), Xh = fp16(v s), Xl =
// fp16(v s - Xh), 1/s.  The row is read once with 16-byte loads into shared
// memory (every load of a thread in flight together), reduced, then split
// from there.  K is a multiple of 4.
enum SplitMode { kPlain = 0, kNorm = 1, kGlu = 2 };

template <int MODE, int NT>
__global__ void __launch_bounds__(NT, 1) split_rows_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                         int64_t K, float eps, __half* __restrict__ xh,
                                                         __half* __restrict__ xl, float* __restrict__ inv_scale) {
  extern __shared__ __align__(16) float vrow[];  // [K]
  grid_dep_launch();  // the matmul after this split may begin its set-up and weight stages
  grid_dep_wait();    // launched as a programmatic dependent: the rows are the previous kernel's
  constexpr int NW = NT / 32;
  __shared__ double dred[NW];
  __shared__ float red[NW];
  const int64_t t = blockIdx.x;
  const int64_t K4 = K >> 2;
  const float4* a4 = reinterpret_cast<const float4*>(A + t * K);
  const float4* b4 = MODE == kGlu ? reinterpret_cast<const float4*>(B + t * K) : nullptr;
  float4* v4 = reinterpret_cast<float4*>(vrow);
  float m = 0.0f;
  double ss = 0.0;
#pragma unroll 4
  for (int64_t i = threadIdx.x; i < K4; i += NT) {
    float4 v = a4[i];
    if (MODE == kGlu) {
      const float4 u = b4[i];
      v.x = (v.x / (1.0f + expf(-v.x))) * u.x;
      v.y = (v.y / (1.0f + expf(-v.y))) * u.y;
      v.z = (v.z / (1.0f + expf(-v.z))) * u.z;
      v.w = (v.w / (1.0f + expf(-v.w))) * u.w;
    }
    if (MODE == kNorm)
      ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    else
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    v4[i] = v;
  }
  if (MODE == kNorm) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) dred[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
    for (int i = 0; i < NW; ++i) tot += dred[i];
    const float nsc = (float)(1.0 / sqrt(tot / (double)K + (double)eps));
    const float4* w4 = reinterpret_cast<const float4*>(B);
#pragma unroll 4
    for (int64_t i = threadIdx.x; i < K4; i += NT) {  // each thread rereads its own entries
      float4 v = v4[i];
      const float4 w = w4[i];
      v.x = v.x * nsc * w.x;
      v.y = v.y * nsc * w.y;
      v.z = v.z * nsc * w.z;
      v.w = v.w * nsc * w.w;
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      v4[i] = v;
    }
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float mx = 0.0f;
  for (int i = 0; i < NW; ++i) mx = fmaxf(mx, red[i]);
  const int e = (int)((__float_as_uint(mx) >> 23) & 0xFFu);  // biased exponent of the max
  // scale 2^(141 - e): max |v| s in [2^14, 2^15); clamped to stay finite
  int se = 141 - e;
  se = se > 100 ? 100 : (se < -100 ? -100 : se);
  const float s = (e == 0 || e == 255) ? 1.0f : exp2f((float)se);
  uint2* h2 = reinterpret_cast<uint2*>(xh + t * K);
  uint2* l2 = reinterpret_cast<uint2*>(xl + t * K);
#pragma unroll 4
  for (int64_t i = threadIdx.x; i < K4; i += NT) {
    const float4 v = v4[i];
    const float y[4] = {v.x * s, v.y * s, v.z * s, v.w * s};
    uint32_t hw[2], lw[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const __half2 hh = __floats2half2_rn(y[2 * k], y[2 * k + 1]);
      const float2 hf = __half22float2(hh);
      const __half2 ll = __floats2half2_rn(y[2 * k] - hf.x, y[2 * k + 1] - hf.y);
      hw[k] = *reinterpret_cast<const uint32_t*>(&hh);
      lw[k] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    h2[i] = make_uint2(hw[0], hw[1]);
    l2[i] = make_uint2(lw[0], lw[1]);
  }
  if (threadIdx.x == 0) inv_scale[t] = 1.0f / (s * kWScale);  // undoes both scalings
}

template <int MODE>
cudaError_t split_rows_launch(const float* A, const float* B, int64_t n, int64_t K, float eps, __half* xh,
                              __half* xl, float* inv, cudaStream_t s) {
  if (K % 4 || K * 4 > 227 * 1024 || ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15))
    return cudaErrorInvalidValue;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = (int)(K * 4);
  if (dev >= 0 && dev < 64 && configured[dev] < smem) {  // dynamic + static above 48 KB needs the opt-in
    cudaError_t e = cudaFuncSetAttribute(split_rows_kernel<MODE, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(split_rows_kernel<MODE, 1024>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = smem;
  }
  // a few hundred rows or more fill the GPU at 256 threads a row; fewer
  // (a batched decode step's session rows) take 1024 threads a row
  const cudaError_t e =
      n >= 256 ? launch_pdl(split_rows_kernel<MODE, 256>, dim3((unsigned)n), dim3(256), (size_t)smem, s, A, B, K, eps, xh, xl, inv)
               : launch_pdl(split_rows_kernel<MODE, 1024>, dim3((unsigned)n), dim3(1024), (size_t)smem, s, A, B, K, eps, xh, xl, inv);
  if (e == cudaSuccess) count_launches(1);
  return e;
}

// OUT[t][r] (+)= sum over the K partitions of the partial sums, in order.
// vec: four consecutive outputs per thread (16-byte accesses; the launcher
// checks that rows, ldo and OUT allow them), else one.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ part, int ks,
                                                            int64_t n, int64_t rows, float* out,
                                                            int64_t ldo, int accumulate, int vec) {
  grid_dep_wait();  // launched as a programmatic dependent of the matmul
  const int64_t total = n * rows;
  if (vec) {
    const int64_t i = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 4;
    if (i >= total) return;
    const int64_t t = i / rows, r = i - t * rows;
    float4 y = __ldcs(reinterpret_cast<const float4*>(part + i));
    for (int p = 1; p < ks; ++p) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(part + (int64_t)p * total + i));
      y.x += v.x;
      y.y += v.y;
      y.z += v.z;
      y.w += v.w;
    }
    float4* o = reinterpret_cast<float4*>(out + t * ldo + r);
    if (accumulate) {
      const float4 c = *o;
      y.x = c.x + y.x;
      y.y = c.y + y.y;
      y.z = c.z + y.z;
      y.w = c.w + y.w;
    }
    *o = y;
    return;
  }
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= total) return;
  const int64_t t = i / rows, r = i - t * rows;
  float y = 0.0f;
  for (int p = 0; p < ks; ++p) y += part[(int64_t)p * total + i];
  float* o = out + t * ldo + r;
  *o = accumulate ? *o + y : y;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_x_map(CUtensorMap* m, const __half* base, int64_t n, int64_t K) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)n};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)TKt, (cuuint32_t)TMt};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Split-K partial sums are bounded by n x kMaxPartRows floats.
constexpr int64_t kMaxPartRows = 9216;

size_t gemm_tc_scratch_bytes(int64_t n, int64_t K) {
  return (((size_t)2 * n * K * sizeof(__half) + (size_t)n * sizeof(float) + 255) & ~(size_t)255) +
         (size_t)n * kMaxPartRows * sizeof(float) + 256;
}

bool gemm_tc_supported(uint32_t type, int64_t K) {
  return K % TKt == 0 && K <= (int64_t)1 << 30 &&
         (type == kQ4_K || type == kQ6_K || type == kQ8_0 || type == kF32);
}

namespace {

template <int TN>
cudaError_t launch_tile(const CUtensorMap& mh, const CUtensorMap& ml, const GemmArgs& g, dim3 grid,
                        cudaStream_t s) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_tc_kernel<TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Tile<TN>::kSmem);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(Tile<TN>::kThreads);
  cfg.dynamicSmemBytes = Tile<TN>::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<TN>, mh, ml, g);
}

// Split-K factor for a tile shape: enough K partitions to fill the GPU
// once, at least 8 stages each, the partial sums (ks x rows per token)
// within the part_rows the scratch holds per token.
int64_t split_k(int64_t tiles, int64_t rows, int64_t K, int nsm, int64_t part_rows) {
  int64_t ks = tiles >= nsm ? 1 : nsm / tiles;
  const int64_t nk = K / TKt;
  if (ks > nk / 8) ks = nk / 8 > 0 ? nk / 8 : 1;
  while (ks > 1 && ks * rows > part_rows) --ks;
  return ks;
}

}  // namespace

namespace {

// One launch over the matrices mat[0..nmat) sharing the input X (n x K):
// the activation split (unless the scratch already holds it), the tile
// height with the least work per SM, split-K (a group's matrices split
// alike), the partial-sum reductions.
cudaError_t launch_group(GemmMat* mat, int nmat, int64_t K, const float* X, int64_t n, bool accumulate,
                         void* scratch, size_t scratch_bytes, cudaStream_t s, bool x_split_ready,
                         const float* glu) {
  if (nmat < 1 || nmat > 3 || n <= 0 || scratch_bytes < gemm_tc_scratch_bytes(n, K) ||
      (reinterpret_cast<uintptr_t>(scratch) & 255) || (nmat > 1 && (glu || accumulate)))
    return cudaErrorInvalidValue;
  for (int i = 0; i < nmat; ++i) {
    if (!gemm_tc_supported(mat[i].type, K) || mat[i].rows <= 0) return cudaErrorInvalidValue;
    if (mat[i].type == kF32 && (mat[i].row_bytes & 15)) return cudaErrorInvalidValue;
  }
  __half* xh = static_cast<__half*>(scratch);
  __half* xl = xh + n * K;
  float* inv = reinterpret_cast<float*>(xl + n * K);
  const size_t part_off = ((size_t)2 * n * K * sizeof(__half) + (size_t)n * sizeof(float) + 255) & ~(size_t)255;
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + part_off);
  // rows of partial sums per token the scratch holds past the split (at least
  // kMaxPartRows; more when the caller passes a larger scratch)
  const int64_t part_rows = (int64_t)((scratch_bytes - part_off) / sizeof(float) / (size_t)n);
  cudaError_t e;
  if (!x_split_ready) {  // else the scratch holds the split of this same X (the caller's promise)
    e = split_rows_launch<kPlain>(X, nullptr, n, K, 0.0f, xh, xl, inv, s);
    if (e != cudaSuccess) return e;
  }
  CUtensorMap mh, ml;
  if (!make_x_map(&mh, xh, n, K) || !make_x_map(&ml, xl, n, K)) return cudaErrorInvalidValue;
  int dev = 0;
  cudaGetDevice(&dev);
  static int sms[64] = {0};
  if (dev >= 0 && dev < 64 && !sms[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = v > 0 ? v : 148;
  }
  const int nsm = (dev >= 0 && dev < 64) ? sms[dev] : 148;
  // tile height: the one with the least work per SM (waves x rows per tile / K partitions)
  const int64_t ttok = (n + TMt - 1) / TMt;
  int64_t best_tn = 128, best_ks = 1;
  double best_cost = 1e30;
  int64_t all_rows = 0;  // partial sums of a group hold every matrix's rows
  for (int i = 0; i < nmat; ++i) all_rows += mat[i].rows;
  for (const int64_t tn : {96, 128, 144}) {
    int64_t tiles = 0;
    for (int i = 0; i < nmat; ++i) tiles += (mat[i].rows + tn - 1) / tn;
    tiles *= ttok;
    const int64_t ks = glu ? 1 : split_k(tiles, all_rows, K, nsm, part_rows);
    const int64_t waves = (tiles * ks + nsm - 1) / nsm;
    const double cost = (double)waves * (double)tn / (double)ks;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best_tn = tn;
      best_ks = ks;
    }
  }
  GemmArgs g;
  int64_t tiles = 0;
  for (int i = 0; i < 3; ++i) {
    g.mat[i] = i < nmat ? mat[i] : mat[0];
    g.mat[i].tiles = (int32_t)((g.mat[i].rows + best_tn - 1) / best_tn);
    if (i < nmat) tiles += g.mat[i].tiles;
  }
  g.nmat = nmat;
  g.K = K;
  g.n = n;
  g.inv_scale = inv;
  g.err = nullptr;
  g.accumulate = accumulate ? 1 : 0;
  g.glu = glu;
  const int64_t ks = best_ks;
  g.ks = (int32_t)ks;
  // split K: matrix i's partial sums [ks][n][rows_i] follow those of the
  // matrices before it
  float* mpart[3] = {part, part, part};
  for (int i = 1; i < nmat; ++i) mpart[i] = mpart[i - 1] + ks * n * mat[i - 1].rows;
  if (ks > 1)
    for (int i = 0; i < nmat; ++i) g.mat[i].out = mpart[i];
  dim3 grid((unsigned)tiles, (unsigned)ttok, (unsigned)ks);
  e = best_tn == 144   ? launch_tile<144>(mh, ml, g, grid, s)
      : best_tn == 128 ? launch_tile<128>(mh, ml, g, grid, s)
                       : launch_tile<96>(mh, ml, g, grid, s);
  if (e == cudaSuccess) count_launches(1);
  if (e != cudaSuccess || ks == 1) return e;
  for (int i = 0; i < nmat; ++i) {
    const int64_t total = n * mat[i].rows;
    const bool vec = (mat[i].rows & 3) == 0 && (mat[i].ldo & 3) == 0 &&
                     (reinterpret_cast<uintptr_t>(mat[i].out) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(mpart[i]) & 15) == 0;
    const int64_t threads = vec ? (total + 3) / 4 : total;
    e = launch_pdl(splitk_reduce_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, s, (const float*)mpart[i],
                   (int)ks, n, mat[i].rows, mat[i].out, mat[i].ldo, accumulate ? 1 : 0, vec ? 1 : 0);
    if (e != cudaSuccess) return e;
    count_launches(1);
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t gemm_tc_launch(uint32_t type, const uint8_t* w, int64_t rows, int64_t K, int64_t row_bytes,
                           const float* X, int64_t n, float* out, int64_t ldo, bool accumulate,
                           void* scratch, size_t scratch_bytes, cudaStream_t s, bool x_split_ready,
                           const float* glu) {
  GemmMat m{w, rows, row_bytes, out, ldo, type, 0};
  return launch_group(&m, 1, K, X, n, accumulate, scratch, scratch_bytes, s, x_split_ready, glu);
}

cudaError_t gemm_tc_split_norm(const float* X, const float* norm_w, float eps, int64_t n, int64_t K,
                               void* scratch, size_t scratch_bytes, cudaStream_t s) {
  if (n <= 0 || K <= 0 || !norm_w || scratch_bytes < gemm_tc_scratch_bytes(n, K) ||
      (reinterpret_cast<uintptr_t>(scratch) & 255))
    return cudaErrorInvalidValue;
  __half* xh = static_cast<__half*>(scratch);
  __half* xl = xh + n * K;
  float* inv = reinterpret_cast<float*>(xl + n * K);
  return split_rows_launch<kNorm>(X, norm_w, n, K, eps, xh, xl, inv, s);
}

cudaError_t gemm_tc_split_glu(const float* gate, const float* up, int64_t n, int64_t K, void* scratch,
                              size_t scratch_bytes, cudaStream_t s) {
  if (n <= 0 || K <= 0 || scratch_bytes < gemm_tc_scratch_bytes(n, K) ||
      (reinterpret_cast<uintptr_t>(scratch) & 255))
    return cudaErrorInvalidValue;
  __half* xh = static_cast<__half*>(scratch);
  __half* xl = xh + n * K;
  float* inv = reinterpret_cast<float*>(xl + n * K);
  return split_rows_launch<kGlu>(gate, up, n, K, 0.0f, xh, xl, inv, s);
}

cudaError_t gemm_tc_launch_group(const GemmGroupMat* mats, int nmat, int64_t K, const float* X, int64_t n,
                                 void* scratch, size_t scratch_bytes, cudaStream_t s, bool x_split_ready) {
  if (nmat < 1 || nmat > 3) return cudaErrorInvalidValue;
  GemmMat m[3];
  for (int i = 0; i < nmat; ++i)
    m[i] = GemmMat{mats[i].w, mats[i].rows, mats[i].row_bytes, mats[i].out, mats[i].ldo, mats[i].type, 0};
  return launch_group(m, nmat, K, X, n, false, scratch, scratch_bytes, s, x_split_ready, nullptr);
}

}  // namespace rpgc
