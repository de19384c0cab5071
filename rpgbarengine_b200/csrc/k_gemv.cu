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
#include "gemv_dev.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

using namespace gemv;

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

__device__ __forceinline__ void consumer_sync(int nc) {
  asm volatile("bar.sync 1, %0;" ::"r"(nc) : "memory");
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
    RingPos rp;
    for (int i = 0; i < first; ++i) rp.advance(NS);
    for (int it = NS; it < n_stages; ++it) {
      mbar_wait(&empty[rp.slot], rp.parity ^ 1u, A.err);
      issue_next(A, P, &cur, stages + (size_t)rp.slot * P.stage_bytes, &desc[rp.slot], &full[rp.slot], pol);
      rp.advance(NS);
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
  RingPos rp;
#pragma unroll 1
  for (int it = 0; it < n_stages; ++it, rp.advance(NS)) {
    const int slot = rp.slot;
    mbar_wait(&full[slot], rp.parity, A.err);
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
      const uint32_t sb = stages32 + (uint32_t)slot * (uint32_t)P.stage_bytes;
      stage_rows<TM>(type, sb + d.off0, L.pair ? sb + d.off1 : sb + d.off0, d.n, s, S, L.pair != 0, rb, u, Ur,
                     uo, act, xf, rbuf + jr0 * Ur, rbuf + (ck_rows + jr0) * Ur);
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
