// k_step.cu -- the persistent decode step: every transformer layer of one
// decode step and the lm_head in ONE kernel, one CTA per SM (cooperative
// launch, so all CTAs are resident together).
//
// Replaces, for decode, the per-token chain of the reference's ForwardStep
// (src/qwen3.cc:119-206, 292-300): per layer RMSNorm -> q/k/v projections ->
// QK-norm + RoPE + KV write + AttentionFromCache -> o projection + residual ->
// RMSNorm -> gate/up + SwiGLU -> down + residual; then the output RMSNorm and
// the lm_head (src/qwen3.cc:208-290).
//
// Phases.  The step is a list of phases (matrix-vector products and one
// attention per layer), each consuming the complete output of the phase
// before it.  A CTA finishes its share of phase p, then increments one step
// counter (release); phase p + 1 starts when the counter reaches
// (p + 1) x grid (acquire; a bounded wait that sets an error flag if it gives
// up).  Every CTA waits for every phase before it signals, so the count
// cannot run ahead of the slowest CTA.
//
// Weight streaming.  The producer warp of each CTA walks the whole step's
// stage program (its rows of every matrix, then its attention tiles) and
// keeps the shared-memory ring full; it never waits for a phase barrier, only
// for free ring slots.  While the consumers stall at a phase boundary (barrier,
// loading and quantising the new input vector), HBM keeps filling the ring,
// so the boundary costs consumer time but no memory time.
//
// Matrix-vector phases use the building blocks of the per-launch GEMV
// (gemv_dev.cuh: activation unit in registers, interleaved 64-element units,
// per-format dp4a unit products, deterministic per-row reduction).
//
// Attention phase.  Work item (kv head kh, split s) of n_kv x splits items
// goes to CTA kh * splits + s: positions [c0, c1) of [0, pos] (the new
// token's row is written into the cache and patched into the shared tile by
// the owner split), online softmax over tiles streamed by the producer, merge
// of 8 warps in shared memory, then the split's partial (o, max, sum per query
// head) goes to global scratch.  A merge phase follows: every CTA combines a
// slice of the attention outputs from their heads' splits in a fixed order.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "attn_dev.cuh"
#include "common.cuh"
#include "gemv_dev.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

using namespace gemv;
using attn::kNegBig;

constexpr int kCWarps = 15;
constexpr int kNC = kCWarps * 32;          // consumer threads
constexpr int kThreads = kNC + 32;         // + one producer warp
constexpr int kMaxStages = 8;
constexpr int kSmemMax = 227 * 1024;       // dynamic shared memory of the one CTA per SM
constexpr int kStageTarget = 32 * 1024;
constexpr int kRedBudget = 16 * 1024;      // partial sums of one reduction chunk (x2 buffers)
constexpr int kAttnWarps = 8;              // warps that score positions
constexpr uint32_t kMaxBarrierPolls = 1u << 22;
constexpr int kRec = 132;                  // floats per attention partial record (16-byte multiple)
constexpr int kMaxItems = 4;               // activation items per consumer thread (K <= 8 * 4 * 480)
constexpr int kMaxNormItems = 2;           // ... with RMSNorm gains (the first round)
constexpr int kPhaseBufOff = 640;          // two phase-table entries in shared memory
constexpr int kCtrStride = 16;             // arrival counters 128 bytes apart (u64 words)
static_assert(kMaxNormItems == 2 && kMaxItems % 2 == 0, "prologue rounds of two items");

struct SLSeg {     // logical segment: one matrix, or a SwiGLU (gate, up) pair
  int32_t rows;
  int32_t first;   // index into seg
  int32_t pair;
  int32_t m;       // rows per stage
  int32_t cs;      // stages per reduction chunk
};

struct alignas(16) PhaseDev {
  int32_t kind;    // 0 matrix-vector, 1 attention
  int32_t cand;    // lm_head: leave the sampler's candidates (LogitCands)
  int32_t nseg, K, U, S, nls, red_floats, half_bytes;
  int32_t deferred;  // 1: every partial of the phase fits the buffers: one reduction at the end
  // tensor parallelism (StepParams::tp_world > 1)
  int32_t x_sum;     // input = xr_prev + the ranks' partial rows of exchange x_xk (rank order)
  int32_t x_xk;
  int32_t xchg;      // 1: partial rows to every rank's inbox; 2: rows to every rank's output copy
  int32_t xchg_k;    // this phase's exchange number in the launch
  GemvSeg seg[3];
  SLSeg ls[3];
  const float* x;
  const float* norm_w;
  const uint64_t* inbox;  // x_sum: this rank's inbox of the exchange [world][K], tagged words
  const float* xr_prev;   // x_sum: the residual before the exchange
  float* xr_next;         // x_sum: the residual after it (each CTA writes its rows)
  void* xdst[kMaxTp];     // xchg: every rank's destination (1: tagged inbox words, 2: floats)
  StepAttn a;
};

struct StepParams {
  const PhaseDev* ph;
  int32_t nph;
  DecodeState* st;
  LogitCands cands;  // val null: none
  const float* rope;
  float eps;
  int32_t n_kv, splits;
  int64_t max_seq;
  float* part;      // [n_kv][splits][G][kRec]: o[128], max, sum, 2 pad
  uint32_t* ctr;    // step counter
  int32_t* err;
  // tensor parallelism: exchanges per launch, this rank's arrival counter
  // (every rank's CTAs add one per exchange) and every rank's (mapped), and
  // this rank's launch counter (grid per launch)
  int32_t tp_world, tp_rank, n_xchg;
  unsigned long long* xctr;    // [kMaxTp][kCtrStride]: one counter per source rank
  unsigned long long* xctr_rank[kMaxTp];
  unsigned long long* launches;
  int32_t stages, stage_bytes, tile_pos, attn_half;
  int32_t ucon_off, lim_off, red_off, ring_off;  // shared-memory carve-up
};

struct SDesc {     // one ring slot's stage, written by the producer before arming
  int64_t r;       // first row / first position
  int32_t n;       // rows / positions
  int32_t ls;      // logical segment (-1: attention tile)
  int32_t last;    // last stage of its logical segment
  uint32_t off0;   // byte offset of row r inside the slot
  uint32_t off1;   // same for the up matrix of a pair
  int32_t phase;
};
static_assert(sizeof(SDesc) == 32, "descriptor size");

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"r"(kNC) : "memory"); }

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// a[i] for i in {0, 1, 2} without indexing (keeps a register array out of
// local memory)
__device__ __forceinline__ int pick3(const int (&a)[3], int i) { return i == 0 ? a[0] : i == 1 ? a[1] : a[2]; }

// Rows [lo, hi) of a segment owned by this CTA (balanced split over the grid).
__device__ __forceinline__ void seg_rows(int32_t rows, int32_t* lo, int32_t* hi) {
  *lo = (int32_t)((uint32_t)rows * blockIdx.x / gridDim.x);
  *hi = (int32_t)((uint32_t)rows * (blockIdx.x + 1) / gridDim.x);
}

// Positions [c0, c1) of attention work item (kh, split) for keys [0, pos].
__device__ __forceinline__ void attn_range(int pos, int splits, int split, int* c0, int* c1) {
  const int L = pos + 1, chunk = (L + splits - 1) / splits;
  *c0 = min(L, split * chunk);
  *c1 = min(L, *c0 + chunk);
}

// Bounded wait until the step counter reaches target (thread 0 of the
// consumers), then release the other consumers.
__device__ __forceinline__ void phase_wait(const StepParams& P, uint32_t target, int tid) {
  if (tid == 0) {
    uint32_t i = 0;
    while (ld_acquire(P.ctr) < target) {
      if (++i > kMaxBarrierPolls) {
        atomicOr(P.err, kErrTimeout);
        break;
      }
      __nanosleep(32);
    }
  }
  csync();
}

// Release add: the barrier orders every consumer's stores of the phase before
// thread 0's release, which is cumulative at GPU scope (no separate fence).
// An exchange phase first adds one to every rank's arrival counter with a
// release at system scope, which covers the CTA's stores to the peers.
template <bool TP>
__device__ __forceinline__ void phase_signal(const StepParams& P, const PhaseDev& ph, int tid) {
  csync();  // every consumer's output of this phase is written
  if (tid == 0) {
    if constexpr (TP) {
      // partial rows (1) carry tags, so their arrival count is relaxed (the
      // readers check every word); the gathered output (2) is plain floats
      // read after the kernel: a release covering the CTA's peer stores
      if (ph.xchg == 1)
        for (int r = 0; r < P.tp_world; ++r)
          asm volatile("red.relaxed.sys.global.add.u64 [%0], 1;" ::"l"(P.xctr_rank[r] + P.tp_rank * kCtrStride)
                       : "memory");
      else if (ph.xchg == 2)
        for (int r = 0; r < P.tp_world; ++r)
          asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(P.xctr_rank[r] + P.tp_rank * kCtrStride)
                       : "memory");
    }
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(P.ctr) : "memory");
  }
}

// Bounded wait (warp 0 of the consumers, lane r watching source rank r's
// counter) until every rank's CTAs have signalled exchange k of launch L,
// then release the other consumers.  The acquires at system scope make the
// peers' stores before their signals visible to this CTA.  A wait gives up
// after ~2 s (a rank that never signals: the error flag is set and the step
// runs on, so the host sees RPGC_E_TIMEOUT), and once any wait of the launch
// has given up the others give up within 256 polls.
constexpr uint32_t kMaxXchgPolls = 1u << 21;
__device__ __forceinline__ void xchg_wait(const StepParams& P, unsigned long long L, int k, int tid) {
  if (tid < 32) {
    const unsigned long long target =
        (L * (unsigned long long)P.n_xchg + (unsigned long long)k + 1ull) * (unsigned long long)gridDim.x;
    bool ok = tid >= P.tp_world;
    uint32_t i = 0;
    for (;;) {
      if (!ok) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(P.xctr + tid * kCtrStride) : "memory");
        ok = v >= target;
      }
      if (__all_sync(0xffffffffu, ok)) break;
      ++i;  // the same count on every lane
      if (i > kMaxXchgPolls || ((i & 255u) == 0 && (*reinterpret_cast<volatile int32_t*>(P.err) & kErrTimeout))) {
        if (tid == 0) atomicOr(P.err, kErrTimeout);
        break;
      }
      __nanosleep(256);
    }
  }
  csync();
}


// ============================================================== producer
__device__ __forceinline__ void slot_acquire(uint64_t* empty, const RingPos& rp, int32_t* err) {
  if (rp.wrapped) mbar_wait_sleep(&empty[rp.slot], rp.parity ^ 1u, err);
}

__device__ void producer(const StepParams& P, uint64_t* full, uint64_t* empty, SDesc* desc,
                         uint8_t* ring, int pos) {
  const uint64_t pol = policy_evict_first();
  const int NS = P.stages;
  RingPos rp;
  for (int p = 0; p < P.nph; ++p) {
    const PhaseDev& ph = P.ph[p];
    if (ph.kind == 0) {
      for (int l = 0; l < ph.nls; ++l) {
        const SLSeg L = ph.ls[l];
        int32_t lo, hi;
        seg_rows(L.rows, &lo, &hi);
        const GemvSeg& G0 = ph.seg[L.first];
        for (int32_t r = lo; r < hi; r += L.m, rp.advance(NS)) {
          const int n = min(L.m, hi - r);
          const int slot = rp.slot;
          slot_acquire(empty, rp, P.err);
          uint8_t* dst = ring + (size_t)slot * P.stage_bytes;
          const uintptr_t s0 = reinterpret_cast<uintptr_t>(G0.w) + (uintptr_t)r * G0.row_bytes;
          const uintptr_t b0 = s0 & ~uintptr_t(15);
          const uint32_t n0 = (uint32_t)(((s0 + (uintptr_t)n * G0.row_bytes + 15) & ~uintptr_t(15)) - b0);
          uintptr_t s1 = 0, b1 = 0;
          uint32_t n1 = 0;
          if (L.pair) {
            const GemvSeg& G1 = ph.seg[L.first + 1];
            s1 = reinterpret_cast<uintptr_t>(G1.w) + (uintptr_t)r * G1.row_bytes;
            b1 = s1 & ~uintptr_t(15);
            n1 = (uint32_t)(((s1 + (uintptr_t)n * G1.row_bytes + 15) & ~uintptr_t(15)) - b1);
          }
          SDesc d;
          d.r = r;
          d.n = n;
          d.ls = l;
          d.last = r + n >= hi;
          d.off0 = (uint32_t)(s0 - b0);
          d.off1 = (uint32_t)ph.half_bytes + (uint32_t)(s1 - b1);
          d.phase = p;
          desc[slot] = d;
          mbar_arrive_expect_tx(&full[slot], n0 + n1);
          bulk_g2s(dst, reinterpret_cast<const void*>(b0), n0, &full[slot], pol);
          if (L.pair) bulk_g2s(dst + ph.half_bytes, reinterpret_cast<const void*>(b1), n1, &full[slot], pol);
        }
      }
    } else if (ph.kind == 1) {
      const int item = (int)blockIdx.x;
      if (item >= P.n_kv * P.splits) continue;
      const int kh = item / P.splits, split = item % P.splits;
      int c0, c1;
      attn_range(pos, P.splits, split, &c0, &c1);
      const float* kb = ph.a.kc + (int64_t)kh * P.max_seq * 128;
      const float* vb = ph.a.vc + (int64_t)kh * P.max_seq * 128;
      for (int t0 = c0; t0 < c1; t0 += P.tile_pos, rp.advance(NS)) {
        const int tn = min(P.tile_pos, c1 - t0);
        const int slot = rp.slot;
        slot_acquire(empty, rp, P.err);
        uint8_t* dst = ring + (size_t)slot * P.stage_bytes;
        SDesc d;
        d.r = t0;
        d.n = tn;
        d.ls = -1;
        d.last = t0 + tn >= c1;
        d.off0 = 0;
        d.off1 = (uint32_t)P.attn_half;
        d.phase = p;
        desc[slot] = d;
        const uint32_t bytes = (uint32_t)tn * 512u;
        mbar_arrive_expect_tx(&full[slot], 2 * bytes);
        bulk_g2s(dst, kb + (int64_t)t0 * 128, bytes, &full[slot], pol);
        bulk_g2s(dst + P.attn_half, vb + (int64_t)t0 * 128, bytes, &full[slot], pol);
      }
    }
  }
}

// ============================================================== consumers
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// Tag of exchange k of launch L (inboxes start at 0xFFFFFFFF, which the
// next 2^32 exchanges do not reach).
__device__ __forceinline__ uint32_t xtag(const StepParams& P, unsigned long long L, int k) {
  return (uint32_t)(L * (unsigned long long)P.n_xchg + (unsigned long long)k + 1ull);
}

// Exchange words: the float's bits in the low half, the exchange's tag in
// the high half, stored and loaded 64 bits at a time at system scope
// (single-copy atomic), so a word showing the expected tag holds its value.
__device__ __forceinline__ void st_xword(void* p, float v, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// Four words at p (16-byte aligned) -> float4; whether every tag is `tag`.
__device__ __forceinline__ bool ld_xwords4(const uint64_t* p, uint32_t tag, float4* v) {
  uint64_t w0, w1, w2, w3;
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w2), "=l"(w3) : "l"(p + 2) : "memory");
  *v = make_float4(__uint_as_float((uint32_t)w0), __uint_as_float((uint32_t)w1), __uint_as_float((uint32_t)w2),
                   __uint_as_float((uint32_t)w3));
  return ((uint32_t)(w0 >> 32) == tag) & ((uint32_t)(w1 >> 32) == tag) & ((uint32_t)(w2 >> 32) == tag) &
         ((uint32_t)(w3 >> 32) == tag);
}

// Elements e..e+3 of an exchange's input: the residual before it plus the
// ranks' partial rows summed in rank order (the same sum on every rank).  A
// partial's words are polled until they carry the exchange's tag (the
// arrival count that let this phase start is relaxed, so a peer's store may
// land after it); bounded, the error flag set on expiry.
__device__ __forceinline__ float4 xsum4(const StepParams& P, const PhaseDev& ph, int e, uint32_t tag) {
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < P.tp_world; ++r) {
    float4 v;
    uint32_t n = 0;
    while (!ld_xwords4(ph.inbox + (size_t)r * ph.K + e, tag, &v)) {
      if (++n > kMaxBarrierPolls || ((n & 255u) == 0 && (*reinterpret_cast<volatile int32_t*>(P.err) & kErrTimeout))) {
        atomicOr(P.err, kErrTimeout);
        break;
      }
      __nanosleep(32);
    }
    s = r ? add4(s, v) : v;
  }
  return add4(__ldcg(reinterpret_cast<const float4*>(ph.xr_prev + e)), s);
}

// The elements of e..e+7 in [lo, hi) into dst.
__device__ __forceinline__ void write_owned(float* dst, int e, float4 a, float4 c, int lo, int hi) {
  const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (e + j >= lo && e + j < hi) dst[e + j] = v[j];
}

// Input vector of a matrix-vector phase.  Thread t quantises items t + NC b
// (two float4 of x each, coalesced); the RMSNorm gains are loaded before the
// phase barrier (they are constant), x after it (written by other CTAs, so
// read through L2), every load of the thread in flight at once.
template <bool TP>
__device__ __forceinline__ void gemv_prologue(const StepParams& P, const PhaseDev& ph, uint32_t target,
                                              unsigned long long L, int tid, int lane, int warp, double* dred,
                                              uint4* lim, float* ucon) {
  const int K = ph.K, NI = K / 8, U = ph.U;
  const bool norm = ph.norm_w != nullptr;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 g0[kMaxNormItems], g1[kMaxNormItems];
#pragma unroll
  for (int b = 0; b < kMaxNormItems; ++b) {
    const int i = b * kNC + tid;
    g0[b] = g1[b] = make_float4(1.f, 1.f, 1.f, 1.f);
    if (norm && i < NI) {
      g0[b] = __ldg(reinterpret_cast<const float4*>(ph.norm_w) + 2 * i);
      g1[b] = __ldg(reinterpret_cast<const float4*>(ph.norm_w) + 2 * i + 1);
    }
  }
  int own_lo = 0, own_hi = 0;  // tensor parallel: this CTA's rows of the new residual
  const bool xs = TP && ph.x_sum;
  if (xs) {
    xchg_wait(P, L, ph.x_xk, tid);
    seg_rows(K, &own_lo, &own_hi);
  } else {
    phase_wait(P, target, tid);
  }
  double ss = 0.0;
  // two items per round, both rounds' loads in flight before any use
#pragma unroll 1
  for (int b0 = 0; b0 < kMaxItems; b0 += 2) {
    if (b0 * kNC >= NI) break;  // uniform
    float4 v0[2], v1[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = (b0 + k) * kNC + tid;
      if (xs) {
        v0[k] = i < NI ? xsum4(P, ph, 8 * i, xtag(P, L, ph.x_xk)) : zero;
        v1[k] = i < NI ? xsum4(P, ph, 8 * i + 4, xtag(P, L, ph.x_xk)) : zero;
      } else {
        v0[k] = i < NI ? __ldcg(reinterpret_cast<const float4*>(ph.x) + 2 * i) : zero;
        v1[k] = i < NI ? __ldcg(reinterpret_cast<const float4*>(ph.x) + 2 * i + 1) : zero;
      }
    }
    if (xs && ph.xr_next) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int i = (b0 + k) * kNC + tid;
        if (i < NI) write_owned(ph.xr_next, 8 * i, v0[k], v1[k], own_lo, own_hi);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int b = b0 + k;
      if (b * kNC >= NI) break;  // uniform
      const int i = b * kNC + tid;
      const float4 a = v0[k], c = v1[k];
      if (norm)
        ss += (double)a.x * a.x + (double)a.y * a.y + (double)a.z * a.z + (double)a.w * a.w +
              (double)c.x * c.x + (double)c.y * c.y + (double)c.z * c.z + (double)c.w * c.w;
      float4 x0 = a, x1 = c;
      if (b0 == 0) {  // gains cover the first two items (host check)
        x0 = make_float4(a.x * g0[k].x, a.y * g0[k].y, a.z * g0[k].z, a.w * g0[k].w);
        x1 = make_float4(c.x * g1[k].x, c.y * g1[k].y, c.z * g1[k].z, c.w * g1[k].w);
      }
      quantize_item(x0, x1, i, i < NI, U, lim, ucon);
    }
  }
  if (norm) {
    ss = warp_sum(ss);
    if (lane == 0) dred[warp] = ss;
  }
  csync();
}

// 1/rms of the phase input from the warps' sums of squares (double, fixed
// order): needed only when the row totals are scaled, so it is taken after
// the matrix work instead of delaying it.
__device__ __forceinline__ float norm_factor(const StepParams& P, const PhaseDev& ph, const double* dred) {
  if (!ph.norm_w) return 1.0f;
  double tot = 0.0;
#pragma unroll
  for (int w = 0; w < kCWarps; ++w) tot += dred[w];
  return 1.0f / sqrtf((float)tot / (float)ph.K + P.eps);
}

// A stored row total: into the segment's output, or for an exchange phase
// into every rank's destination (plain stores, peers' memory included).
template <bool TP>
__device__ __forceinline__ void out_row(const StepParams& P, const PhaseDev& ph, const GemvSeg& G, int32_t row,
                                        float t, unsigned long long L) {
  if (TP && ph.xchg == 1) {
    const uint32_t tag = xtag(P, L, ph.xchg_k);
    for (int r = 0; r < P.tp_world; ++r) st_xword(static_cast<uint64_t*>(ph.xdst[r]) + row, t, tag);
  } else if (TP && ph.xchg == 2) {
    for (int r = 0; r < P.tp_world; ++r) static_cast<float*>(ph.xdst[r])[row] = t;
  } else {
    G.out[row] = t;
  }
}

template <uint32_t TM, bool TP>
__device__ __forceinline__ void gemv_phase(const StepParams& P, const PhaseDev& ph, uint32_t target,
                                           unsigned long long launch, RingPos* rpp, uint64_t* full, uint64_t* empty,
                                           const SDesc* desc, uint32_t ring32, double* dred, uint4* lim, float* ucon,
                                           float* red, int tid, int lane, int warp) {
  gemv_prologue<TP>(P, ph, target, launch, tid, lane, warp, dred, lim, ucon);
  const int U = ph.U, S = ph.S, Ur = U | 1, NS = P.stages;
  // this CTA's rows of each logical segment, once per phase
  int slo[3] = {0, 0, 0}, sn[3] = {0, 0, 0};
#pragma unroll
  for (int l = 0; l < 3; ++l)
    if (l < ph.nls) {
      int32_t lo, hi;
      seg_rows(ph.ls[l].rows, &lo, &hi);
      slo[l] = lo;
      sn[l] = hi - lo;
    }
  const int u = tid % U, s = tid / U;
  const bool busy = s < S;
  const UnitOff uo = unit_offsets(u);
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
  RingPos rp = *rpp;
  const uint32_t sbytes = (uint32_t)P.stage_bytes;
  // rows j (stage-relative) of one stage into partial slots p0 (+ j * Ur)
  // and, for the second row, p1
  auto rows = [&](const SDesc& d, int slot, const SLSeg& L, uint32_t type, int rb, float* p0, float* p1) {
    if (!busy) return;
    const uint32_t sb = ring32 + (uint32_t)slot * sbytes;
    stage_rows<TM>(type, sb + d.off0, L.pair ? sb + d.off1 : sb + d.off0, d.n, s, S, L.pair != 0, rb, u, Ur, uo,
                   act, nullptr, p0, p1);
  };
  // row total of partial row pp over tpr threads (4, 8 or 16 adjacent
  // lanes), fixed order: deterministic for a phase shape
  auto row_total = [&](const float* pp, int q, bool live, int tpr, float nscale) {
    float t = 0.0f;
    if (live) {
#pragma unroll 4
      for (int v = q; v < U; v += tpr) t += pp[v];
    }
    for (int m = 1; m < tpr; m <<= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
    return t * nscale;
  };
  if (ph.deferred) {
    int base = 0;
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      if (l >= ph.nls) break;
      const SLSeg L = ph.ls[l];
      const int lo = slo[l], nrows = sn[l];
      const GemvSeg G = ph.seg[L.first];
      const int nst = (nrows + L.m - 1) / L.m;
#pragma unroll 1
      for (int k = 0; k < nst; ++k, rp.advance(NS)) {
        const int slot = rp.slot;
        mbar_wait(&full[slot], rp.parity, P.err);
        const SDesc d = desc[slot];
        const int jr0 = (int)d.r - lo;
        rows(d, slot, L, G.type, (int)G.row_bytes, red + base + jr0 * Ur, red + base + (nrows + jr0) * Ur);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
      base += nrows * (L.pair + 1) * Ur;
    }
    // one reduction over every segment's rows: sum sid of segment l is row
    // (pair ? sid / 2 : sid), half (pair ? sid % 2 : 0); tpr threads per sum
    // (the most, up to 16, that still take every sum in one pass over the
    // consumers: measured, a second pass costs more than longer serial sums)
    int total = 0;
#pragma unroll
    for (int l = 0; l < 3; ++l)
      if (l < ph.nls) total += sn[l] * (ph.ls[l].pair + 1);
    const int lg = total * 16 <= kNC ? 4 : total * 8 <= kNC ? 3 : total * 4 <= kNC ? 2 : total * 2 <= kNC ? 1 : 0,
              tpr = 1 << lg;
    struct Sum {
      int l, j, h, bse;
      bool live;
    };
    auto locate = [&](int sid) {
      Sum r{0, 0, 0, 0, false};
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        if (r.live || l >= ph.nls) continue;
        const int pr = ph.ls[l].pair, n = sn[l] * (pr + 1);
        if (sid < n) {
          r = Sum{l, pr ? sid >> 1 : sid, pr ? sid & 1 : 0, r.bse, true};
        } else {
          sid -= n;
          r.bse += n * Ur;
        }
      }
      return r;
    };
    // the residual rows this thread adds to, loaded before the barrier
    float resid = 0.0f;
    {
      const Sum a = locate(tid >> lg);
      if (a.live && (tid & (tpr - 1)) == 0 && a.h == 0) {
        const SLSeg& L = ph.ls[a.l];
        const GemvSeg& G = ph.seg[L.first];
        if (!L.pair && G.mode == kAdd) resid = __ldcg(G.out + pick3(slo, a.l) + a.j);
      }
    }
    const float nscale = norm_factor(P, ph, dred);
    csync();
#pragma unroll 1
    for (int b0 = 0; b0 < total * tpr; b0 += kNC) {
      const int idx = b0 + tid, q = idx & (tpr - 1);
      const Sum a = locate(idx >> lg);
      const int ll = a.live ? a.l : 0;
      const SLSeg& L = ph.ls[ll];
      const float t = row_total(red + a.bse + (a.h * pick3(sn, ll) + a.j) * Ur, q, a.live, tpr, nscale);
      const float other = __shfl_xor_sync(0xffffffffu, t, tpr);  // up total for a pair's gate lanes
      if (a.live && q == 0 && a.h == 0) {
        const GemvSeg& G = ph.seg[L.first];
        const int32_t row = pick3(slo, ll) + a.j;
        if (L.pair) ph.seg[L.first + 1].out[row] = silu_mul(t, other);
        else if (G.mode == kAdd) G.out[row] = (b0 == 0 ? resid : __ldcg(G.out + row)) + t;
        else out_row<TP>(P, ph, G, row, t, launch);
      }
    }
    *rpp = rp;
    return;
  }
  const float nscale = norm_factor(P, ph, dred);
#pragma unroll 1
  for (int l = 0; l < ph.nls; ++l) {
    const SLSeg L = ph.ls[l];
    const int32_t lo = pick3(slo, l), hi = lo + pick3(sn, l);
    const GemvSeg G = ph.seg[L.first];
    float* up_out = L.pair ? ph.seg[L.first + 1].out : nullptr;
    const int rb = (int)G.row_bytes, ck_rows = L.cs * L.m;
    const int nst = (hi - lo + L.m - 1) / L.m;
    int chunk0 = 0, cbuf = 0;
    int32_t chunk_r0 = lo;
#pragma unroll 1
    for (int k = 0; k < nst; ++k, rp.advance(NS)) {
      const int slot = rp.slot;
      mbar_wait(&full[slot], rp.parity, P.err);
      const SDesc d = desc[slot];
      if (k == chunk0) chunk_r0 = (int32_t)d.r;
      const int jr0 = (k - chunk0) * L.m;
      float* rbuf = red + cbuf * ph.red_floats;
      rows(d, slot, L, G.type, rb, rbuf + jr0 * Ur, rbuf + (ck_rows + jr0) * Ur);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (!d.last && k + 1 - chunk0 < L.cs) continue;
      // chunk complete: 4 threads per row total, fixed order (deterministic)
      csync();
      const int rows = jr0 + d.n, nsum = rows * (L.pair + 1);
#pragma unroll 1
      for (int b0 = 0; b0 < 4 * nsum; b0 += kNC) {
        const int idx = b0 + tid, q = idx & 3, sid = idx >> 2;
        const int j = L.pair ? sid >> 1 : sid, h = L.pair ? sid & 1 : 0;
        const float t = row_total(rbuf + (h * ck_rows + j) * Ur, q, sid < nsum, 4, nscale);
        const float other = __shfl_xor_sync(0xffffffffu, t, 4);
        if (sid < nsum && q == 0 && h == 0) {
          const int32_t row = chunk_r0 + j;
          if (L.pair) up_out[row] = silu_mul(t, other);
          else if (G.mode == kAdd) G.out[row] += t;
          else out_row<TP>(P, ph, G, row, t, launch);
        }
      }
      chunk0 = k + 1;
      cbuf ^= 1;
    }
  }
  *rpp = rp;
}

// Attention phase of one layer for a group of G query heads per kv head.
template <int G>
__device__ __forceinline__ void attn_phase(const StepParams& P, const PhaseDev& ph, uint32_t target, RingPos* rpp, uint64_t* full,
                                           uint64_t* empty, const SDesc* desc, uint8_t* ring, float* scratch,
                                           int pos, int tid, int lane, int warp) {
  constexpr int PB = 32 / G;
  const StepAttn& A = ph.a;
  const int item = (int)blockIdx.x, NS = P.stages;
  const bool has_item = item < P.n_kv * P.splits;
  const int kh = has_item ? item / P.splits : 0, split = has_item ? item % P.splits : 0;
  int c0 = 0, c1 = 0;
  if (has_item) attn_range(pos, P.splits, split, &c0, &c1);
  const bool owner = has_item && c0 <= pos && pos < c1;
  const float* cs = P.rope + (int64_t)pos * 128;
  // scratch: qs[G][128] | wo[kAttnWarps][G][128] | wm[kAttnWarps][G] | wl[kAttnWarps][G] | kv_new[2][128]
  // (the new token's k and v are kept in shared memory, not in registers
  // across the tile loop, where they would push the kernel into spills)
  float* qs = scratch;
  float* wo = qs + G * 128;
  float* wm = wo + kAttnWarps * G * 128;
  float* wl = wm + kAttnWarps * G;
  float* kv_new = wl + kAttnWarps * G;  // [2][128]: the new token's k and v (owner warp)
  // constants of the QK-norm and the rotation, before the phase barrier
  const float4 rc = __ldg(reinterpret_cast<const float4*>(cs + ((4 * lane) & 63)));
  const float4 rs = __ldg(reinterpret_cast<const float4*>(cs + 64 + ((4 * lane) & 63)));
  const float4 gq = __ldg(reinterpret_cast<const float4*>(A.q_norm) + lane);
  const float4 gk = __ldg(reinterpret_cast<const float4*>(A.k_norm) + lane);
  phase_wait(P, target, tid);
  if (has_item) {
    if (warp < G) {
      float4 v = __ldcg(reinterpret_cast<const float4*>(A.q + (kh * G + warp) * 128) + lane);
      v = attn::norm_rope_head_pre(v, gq, rc, rs, P.eps, lane);
      reinterpret_cast<float4*>(qs + warp * 128)[lane] = v;
    }
    if (owner && warp == kAttnWarps) {  // the new token's k and v: into the cache
      float4 knew = __ldcg(reinterpret_cast<const float4*>(A.k_new + kh * 128) + lane);
      knew = attn::norm_rope_head_pre(knew, gk, rc, rs, P.eps, lane);
      const float4 vnew = __ldcg(reinterpret_cast<const float4*>(A.v_new + kh * 128) + lane);
      reinterpret_cast<float4*>(kv_new)[lane] = knew;
      reinterpret_cast<float4*>(kv_new + 128)[lane] = vnew;
      const int64_t off = ((int64_t)kh * P.max_seq + pos) * 128 + 4 * lane;
      *reinterpret_cast<float4*>(A.kc + off) = knew;
      *reinterpret_cast<float4*>(A.vc + off) = vnew;
    }
  }
  csync();
  const float scale = 1.0f / sqrtf(128.0f);
  float4 q[G], o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    q[g] = reinterpret_cast<const float4*>(qs + g * 128)[lane];
    o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mh = kNegBig, lh = 0.0f;
  const int gl = lane / PB, jl = lane % PB;
  RingPos rp = *rpp;
  for (int t0 = c0; t0 < c1; t0 += P.tile_pos, rp.advance(NS)) {
    const int slot = rp.slot;
    mbar_wait(&full[slot], rp.parity, P.err);
    const int tn = min(P.tile_pos, c1 - t0);
    float* Ks = reinterpret_cast<float*>(ring + (size_t)slot * P.stage_bytes);
    float* Vs = reinterpret_cast<float*>(ring + (size_t)slot * P.stage_bytes + P.attn_half);
    if (owner && warp == kAttnWarps && pos >= t0 && pos < t0 + tn) {
      reinterpret_cast<float4*>(Ks + (pos - t0) * 128)[lane] = reinterpret_cast<const float4*>(kv_new)[lane];
      reinterpret_cast<float4*>(Vs + (pos - t0) * 128)[lane] = reinterpret_cast<const float4*>(kv_new + 128)[lane];
    }
    if (owner) csync();  // the patched row is visible to every scoring warp (CTA-uniform condition)
    if (warp < kAttnWarps) {
      for (int pb = warp * PB; pb < tn; pb += kAttnWarps * PB) {
        float val[32];
#pragma unroll
        for (int j = 0; j < PB; ++j) {
          const float4 k = pb + j < tn ? reinterpret_cast<const float4*>(Ks + (pb + j) * 128)[lane]
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int g = 0; g < G; ++g) val[g * PB + j] = attn::dot4(q[g], k);
        }
        const bool valid = pb + jl < tn;
        const float tr = attn::transpose_reduce(val, lane);
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
            const float pj = __shfl_sync(0xffffffffu, pe, g * PB + j);
            o[g].x += pj * v.x;
            o[g].y += pj * v.y;
            o[g].z += pj * v.z;
            o[g].w += pj * v.w;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  *rpp = rp;
  // ---- merge the scoring warps of this CTA into the split's partial
  if (warp < kAttnWarps) {
#pragma unroll
    for (int g = 0; g < G; ++g) reinterpret_cast<float4*>(wo + (warp * G + g) * 128)[lane] = o[g];
    if (jl == 0) {
      wm[warp * G + gl] = mh;
      wl[warp * G + gl] = lh;
    }
  }
  csync();
  float* mypart = P.part + ((int64_t)kh * P.splits + split) * (G * kRec);
  if (has_item) {
    for (int idx = tid; idx < G * 128; idx += kNC) {
      const int g = idx >> 7, d = idx & 127;
      float M = kNegBig;
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w * G + g]);
      float O = 0.0f, Ls = 0.0f;
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = expf(wm[w * G + g] - M);
        O += wo[(w * G + g) * 128 + d] * f;
        Ls += wl[w * G + g] * f;
      }
      mypart[g * kRec + d] = O;
      if (d == 0) {
        mypart[g * kRec + 128] = M;
        mypart[g * kRec + 129] = Ls;
      }
    }
  }
}

// Merge phase after an attention phase: every split of a kv head has written
// its partial (o, max, sum per query head), so output o of the n_kv * G * 128
// attention outputs is combined from its head's splits in a fixed order
// (max, then the rescaled sums).  Each CTA takes a contiguous slice of the
// outputs; its loads are all independent (one L2 round trip).
template <int G>
__device__ __noinline__ void merge_phase(const StepParams& P, const PhaseDev& ph, uint32_t target, int tid,
                                         float* scratch) {
  phase_wait(P, target, tid);
  const int nout = P.n_kv * G * 128, S = P.splits;
  const int o0 = (int)((int64_t)nout * blockIdx.x / gridDim.x), o1 = (int)((int64_t)nout * (blockIdx.x + 1) / gridDim.x);
  const int n_o = o1 - o0;
  // stage (output, split) -> (o, max, sum) with every load in flight at once
  // (one L2 round trip), then combine from shared memory
#pragma unroll 1
  for (int i = tid; i < n_o * S; i += kNC) {
    const int o = o0 + i / S, r = i % S;
    const int kh = o / (G * 128), g = (o >> 7) % G, d = o & 127;
    const float* rp = P.part + ((int64_t)kh * S + r) * (G * kRec) + g * kRec;
    scratch[3 * i] = __ldcg(rp + d);
    scratch[3 * i + 1] = __ldcg(rp + 128);
    scratch[3 * i + 2] = __ldcg(rp + 129);
  }
  csync();
#pragma unroll 1
  for (int i = tid; i < n_o; i += kNC) {
    const float* sp = scratch + 3 * i * S;
    float M = kNegBig;
    for (int r = 0; r < S; ++r) M = fmaxf(M, sp[3 * r + 1]);
    float O = 0.0f, Ls = 0.0f;
    for (int r = 0; r < S; ++r) {
      const float f = expf(sp[3 * r + 1] - M);
      O += sp[3 * r] * f;
      Ls += sp[3 * r + 2] * f;
    }
    const int o = o0 + i, kh = o / (G * 128), g = (o >> 7) % G, d = o & 127;
    ph.a.out[(kh * G + g) * 128 + d] = O / Ls;
  }
}

// ------------------------------------------------- sampler candidates
// 64-bit order key of a logit: larger value first, ties to the lower index.
// Key 0 is padding (a NaN is reported by the CTA instead of listed).
__device__ __forceinline__ uint64_t cand_key(float v, int32_t i) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)k << 32) | (uint32_t)(0x7FFFFFFF - i);
}
__device__ __forceinline__ float cand_value(uint64_t key) {
  const uint32_t k = (uint32_t)(key >> 32);
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
__device__ __forceinline__ int32_t cand_index(uint64_t key) { return 0x7FFFFFFF - (int32_t)(uint32_t)key; }

__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), m);
  return ((uint64_t)hi << 32) | lo;
}
// One compare-exchange stage (block size k, distance j) of a bitonic network
// over the warp's 32 keys, descending overall.
__device__ __forceinline__ uint64_t bitonic_step(uint64_t key, int lane, int k, int j) {
  const uint64_t o = shfl_xor64(key, j);
  const bool keep_max = ((lane & j) == 0) == ((lane & k) == 0);
  return keep_max ? (key > o ? key : o) : (key < o ? key : o);
}
__device__ __forceinline__ uint64_t warp_sort_desc(uint64_t key, int lane) {
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) key = bitonic_step(key, lane, k, j);
  return key;
}
// The 32 largest of two descending lists, descending: the elementwise max
// against the other list reversed is bitonic; one merge network sorts it.
__device__ __forceinline__ uint64_t warp_merge_desc(uint64_t a, uint64_t b, int lane) {
  const uint32_t lo = __shfl_sync(0xffffffffu, (uint32_t)b, 31 - lane);
  const uint32_t hi = __shfl_sync(0xffffffffu, (uint32_t)(b >> 32), 31 - lane);
  const uint64_t br = ((uint64_t)hi << 32) | lo;
  uint64_t key = a > br ? a : br;
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) key = bitonic_step(key, lane, 32, j);
  return key;
}

// After the lm_head phase: this CTA's rows of the logits -> the first index
// of its maximum and, when the sampler draws with 1 < top_k <= kCandK, its
// kCandK largest (ties to the lower index) in index order.  Sets
// st->cand_ok; a NaN among the rows marks max_idx -2 (the sampler then
// sweeps the whole vocabulary, as it does for the options this skips).
__device__ __noinline__ void cand_phase(const StepParams& P, const PhaseDev& ph, int lane, int warp,
                                        uint64_t* lists, int* flags) {
  DecodeState* st = P.st;
  const int mode = !st ? 0 : !(st->temperature > 0.0f) ? 1 : (st->top_k > 1 && st->top_k <= kCandK) ? 2 : 0;
  const int c = (int)blockIdx.x;
  if (mode == 0 || c >= P.cands.ctas) return;  // uniform over the CTA
  csync();  // the phase's row totals are stored
  const GemvSeg& G = ph.seg[0];
  int32_t lo, hi;
  seg_rows((int32_t)G.rows, &lo, &hi);
  const int R = hi - lo;
  const int w0 = lo + (int)((int64_t)R * warp / kCWarps), w1 = lo + (int)((int64_t)R * (warp + 1) / kCWarps);
  uint64_t top = 0;
  bool nan = false;
  if (mode == 1) {  // the maximum only
#pragma unroll 1
    for (int r = w0 + lane; r < w1; r += 32) {
      const float v = __ldcg(G.out + r);
      nan |= v != v;
      const uint64_t k = v != v ? 0ull : cand_key(v, r);
      top = k > top ? k : top;
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      const uint64_t o = shfl_xor64(top, m);
      top = o > top ? o : top;
    }
  } else {
#pragma unroll 1
    for (int r0 = w0; r0 < w1; r0 += 32) {  // warp-uniform batches of 32 rows
      const int r = r0 + lane;
      const float v = r < w1 ? __ldcg(G.out + r) : 0.0f;
      nan |= r < w1 && v != v;
      uint64_t k = (r < w1 && v == v) ? cand_key(v, r) : 0ull;
      k = warp_sort_desc(k, lane);
      top = r0 == w0 ? k : warp_merge_desc(top, k, lane);
    }
  }
  nan = __any_sync(0xffffffffu, nan);
  lists[warp * 32 + lane] = top;
  if (lane == 0) flags[warp] = nan;
  csync();
  if (mode == 2) {  // merge the warps' lists pairwise: 15 -> 8 -> 4 -> 2 -> 1
    int count = kCWarps;
#pragma unroll 1
    for (int step = 8; step >= 1; step >>= 1) {
      if (warp < step && warp + step < count) {
        const uint64_t m = warp_merge_desc(lists[warp * 32 + lane], lists[(warp + step) * 32 + lane], lane);
        __syncwarp();
        lists[warp * 32 + lane] = m;
      }
      count = step;
      csync();
    }
  }
  if (warp == 0) {
    bool any_nan = false;
    uint64_t best = 0;
#pragma unroll 1
    for (int w = 0; w < kCWarps; ++w) {
      any_nan |= flags[w] != 0;
      if (mode == 1) best = lists[w * 32] > best ? lists[w * 32] : best;
    }
    if (mode == 2) best = lists[0];
    if (lane == 0) {
      P.cands.max_val[c] = best ? cand_value(best) : 0.0f;
      P.cands.max_idx[c] = any_nan ? -2 : best ? cand_index(best) : -1;
    }
    if (mode == 2) {
      // the list in index order: sort (index, value bits) ascending
      const uint64_t k = lists[lane];
      const uint64_t key2 = k ? ((uint64_t)(uint32_t)cand_index(k) << 32) | __float_as_uint(cand_value(k))
                              : ~0ull;
      const uint64_t sorted = ~warp_sort_desc(~key2, lane);
      const bool pad = sorted == ~0ull;
      P.cands.val[c * kCandK + lane] = pad ? 0.0f : __uint_as_float((uint32_t)sorted);
      P.cands.idx[c * kCandK + lane] = pad ? -1 : (int32_t)(sorted >> 32);
    }
    if (lane == 0) st->cand_ok = mode;
  }
}

template <uint32_t TM, int G, bool TP>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);             // [kMaxStages]
  uint64_t* empty = full + kMaxStages;                            // [kMaxStages]
  SDesc* desc = reinterpret_cast<SDesc*>(smem + 128);             // [kMaxStages]
  double* dred = reinterpret_cast<double*>(smem + 384);           // [16]
  // the consumers' copies of the phase table entries: phase p in pbuf[p & 1]
  // (the table lives in global memory, and with the ring taking nearly all of
  // the SM's shared memory L1 is too small to keep it)
  PhaseDev* pbuf = reinterpret_cast<PhaseDev*>(smem + kPhaseBufOff);
  float* ucon = reinterpret_cast<float*>(smem + P.ucon_off);
  uint4* lim = reinterpret_cast<uint4*>(smem + P.lim_off);
  float* red = reinterpret_cast<float*>(smem + P.red_off);
  float* scratch = reinterpret_cast<float*>(smem + P.lim_off);   // attention (aliases lim, red)
  uint8_t* ring = smem + P.ring_off;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const DecodeState* st = P.st;
  if (st && !st->active) return;  // every CTA leaves
  const int pos = st ? st->pos : 0;
  if (tid == kNC) {
    for (int i = 0; i < P.stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (tid >= kNC) {
    if (tid == kNC) producer(P, full, empty, desc, ring, pos);
    return;
  }
  const uint32_t ring32 = smem_u32(ring);
  RingPos it;
  constexpr int kPhaseChunks = (int)(sizeof(PhaseDev) / 16);
  if (tid < kPhaseChunks) {
    cp_async16(reinterpret_cast<uint4*>(pbuf) + tid, reinterpret_cast<const uint4*>(P.ph) + tid);
    cp_async_wait_all();
  }
  // tensor parallelism: this launch's number (every CTA of a launch adds
  // one, and a launch starts after the previous one ended)
  unsigned long long* launch_s = reinterpret_cast<unsigned long long*>(smem + 512);
  if constexpr (TP) {
    if (tid == 0) *launch_s = atomicAdd(P.launches, 1ull) / gridDim.x;
  }
  csync();
  const unsigned long long L = TP ? *launch_s : 0ull;
#pragma unroll 1
  for (int p = 0; p < P.nph; ++p) {
    const PhaseDev& ph = pbuf[p & 1];
    const uint32_t target = (uint32_t)p * gridDim.x;
    // the next phase's entry arrives while this phase runs; the copy is
    // waited for before this phase's closing barrier
    if (tid < kPhaseChunks && p + 1 < P.nph)
      cp_async16(reinterpret_cast<uint4*>(pbuf + ((p + 1) & 1)) + tid,
                 reinterpret_cast<const uint4*>(P.ph + p + 1) + tid);
    if (ph.kind == 0) {
      gemv_phase<TM, TP>(P, ph, target, L, &it, full, empty, desc, ring32, dred, lim, ucon, red, tid, lane, warp);
      if (ph.cand && P.cands.val)  // the phase's reduction buffers are free again
        cand_phase(P, ph, lane, warp, reinterpret_cast<uint64_t*>(red), reinterpret_cast<int*>(lim));
    } else if (ph.kind == 1) {
      attn_phase<G>(P, ph, target, &it, full, empty, desc, ring, scratch, pos, tid, lane, warp);
    } else {
      merge_phase<G>(P, ph, target, tid, scratch);
    }
    if (tid < kPhaseChunks) cp_async_wait_all();
    phase_signal<TP>(P, ph, tid);
  }
  // tensor parallelism: the last exchange (every rank's rows of the output)
  // has arrived before the kernel ends, so the launches after it read it whole
  if constexpr (TP) {
    if (blockIdx.x == 0) xchg_wait(P, L, P.n_xchg - 1, tid);
  }
}

// ------------------------------------------------------------------ host
constexpr uint32_t type_mask(uint32_t t) {
  return t == kQ4_K ? kMQ4K : t == kQ6_K ? kMQ6K : t == kQ8_0 ? kMQ80 : 0;
}

struct Geometry {
  int stage_bytes = 0, stages = 0, tile_pos = 0, attn_half = 0;
  int ucon_off = 0, lim_off = 0, red_off = 0, ring_off = 0, smem = 0;
};

bool plan_gemv(const StepGemv& g, PhaseDev* d, int* slot_need) {
  if (g.nseg < 1 || g.nseg > 3 || g.K <= 0 || g.K % 128 != 0) return false;
  const int U = g.K / 64;
  if (U > kNC) return false;
  d->kind = 0;
  d->nseg = g.nseg;
  d->K = g.K;
  d->U = U;
  d->S = kNC / U;
  d->x = g.x;
  d->norm_w = g.norm_w;
  d->nls = 0;
  int half = 0, red = 0, need = 0;
  for (int i = 0; i < g.nseg; ++i) {
    const GemvSeg& G = g.seg[i];
    d->seg[i] = G;
    int be, bb;
    switch (G.type) {
      case kQ4_K: be = 256; bb = 144; break;
      case kQ6_K: be = 256; bb = 210; break;
      case kQ8_0: be = 32; bb = 34; break;
      default: return false;
    }
    if (g.K % be != 0 || (int64_t)(g.K / be) * bb != G.row_bytes) return false;
    if (reinterpret_cast<uintptr_t>(G.w) & 15) return false;
    if (G.rows <= 0 || G.rows > (int64_t)(0xFFFFFFFFu / 1024)) return false;
    const bool up_of_pair = i > 0 && g.seg[i - 1].mode == kSwiGLU;
    if (up_of_pair) {
      if (G.rows != g.seg[i - 1].rows || G.type != g.seg[i - 1].type) return false;
      continue;
    }
    SLSeg& L = d->ls[d->nls++];
    L.rows = (int32_t)G.rows;
    L.first = i;
    L.pair = G.mode == kSwiGLU ? 1 : 0;
    const int64_t per_round = (int64_t)d->S * G.row_bytes * 2;
    int64_t rounds = kStageTarget / per_round;
    if (rounds < 1) rounds = 1;
    L.m = (int32_t)(rounds * d->S * (L.pair ? 1 : 2));
    const int slot = (int)(((int64_t)L.m * G.row_bytes + 32 + 127) & ~int64_t(127));
    if (L.pair) half = std::max(half, slot);
    need = std::max(need, slot * (L.pair + 1));
    const int per_stage = L.m * (U | 1) * (L.pair + 1);
    int cs = kRedBudget / (4 * per_stage);
    if (cs < 1) cs = 1;
    L.cs = cs;
    red = std::max(red, cs * per_stage);
  }
  if (g.seg[g.nseg - 1].mode == kSwiGLU) return false;
  if (g.K / 8 > kMaxItems * kNC) return false;
  if (g.norm_w && g.K / 8 > kMaxNormItems * kNC) return false;
  d->red_floats = red;
  d->deferred = 0;
  d->half_bytes = half;
  *slot_need = need;
  return true;
}

int sms_of(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <uint32_t TM, int G, bool TP>
cudaError_t launch_g(const StepParams& p, int grid, int smem, cudaStream_t s) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && configured[dev] < smem) {
    cudaError_t e = cudaFuncSetAttribute(step_kernel<TM, G, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, step_kernel<TM, G, TP>, p);
  if (e == cudaSuccess) count_launches(1);
  return e;
}

// Whether one CTA of the instantiation fits an SM with `smem` bytes.
template <uint32_t TM, int G, bool TP>
bool fits_g(int smem) {
  if (cudaFuncSetAttribute(step_kernel<TM, G, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, step_kernel<TM, G, TP>, kThreads, smem) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return n >= 1;
}

template <uint32_t TM, bool TP>
bool fits_tm(int G, int smem) {
  switch (G) {
    case 1: return fits_g<TM, 1, TP>(smem);
    case 2: return fits_g<TM, 2, TP>(smem);
    case 4: return fits_g<TM, 4, TP>(smem);
    case 8: return fits_g<TM, 8, TP>(smem);
    default: return false;
  }
}

// Instantiations: one per block-type mix and query group; the
// tensor-parallel kernel (exchanges compiled in) for all-Q8_0 models and for
// any mix.
bool fits(uint32_t mask, int G, int smem, bool tp) {
  if (tp) return mask == kMQ80 ? fits_tm<kMQ80, true>(G, smem) : fits_tm<kMQ4K | kMQ6K | kMQ80, true>(G, smem);
  if ((mask & ~(kMQ4K | kMQ6K)) == 0) return fits_tm<kMQ4K | kMQ6K, false>(G, smem);
  if (mask == kMQ80) return fits_tm<kMQ80, false>(G, smem);
  return fits_tm<kMQ4K | kMQ6K | kMQ80, false>(G, smem);
}

template <uint32_t TM, bool TP>
cudaError_t launch_tm(const StepParams& p, int G, int grid, int smem, cudaStream_t s) {
  switch (G) {
    case 1: return launch_g<TM, 1, TP>(p, grid, smem, s);
    case 2: return launch_g<TM, 2, TP>(p, grid, smem, s);
    case 4: return launch_g<TM, 4, TP>(p, grid, smem, s);
    case 8: return launch_g<TM, 8, TP>(p, grid, smem, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

struct StepPlan {
  PhaseDev* dev = nullptr;  // device phase table
  int nph = 0;
  Geometry geo;
  uint32_t mask = 0;
  int grid = 0, n_kv = 0, G = 0, splits = 0;
  int64_t max_seq = 0;
  // tensor parallelism: the arena every rank maps (arrival counter, launch
  // counter, two exchange inboxes [world][hidden], two residual buffers), the
  // phase table kept on the host until every rank's arena is bound
  StepTp tp{0, 1, 0, 0};
  uint8_t* arena = nullptr;
  int n_xchg = 0;
  std::vector<PhaseDev> table;
  unsigned long long* xctr_rank[kMaxTp] = {};
  bool bound = true;
};

namespace {
// arrival counters (one per source rank, 128 bytes apart) at 0, launch
// counter at kMaxTp x 128
constexpr size_t kLaunchOff = (size_t)kMaxTp * kCtrStride * 8;
constexpr size_t kArenaHead = kLaunchOff + 256;
size_t inbox_off(const StepTp& t, int slot) { return kArenaHead + (size_t)slot * t.world * t.hidden * 8; }
size_t xr_off(const StepTp& t, int i) { return inbox_off(t, 2) + (size_t)i * t.hidden * 4; }
size_t arena_bytes(const StepTp& t) { return xr_off(t, 2); }
}  // namespace

size_t step_part_floats(const StepPlan* p) {
  return p ? (size_t)p->n_kv * p->splits * p->G * kRec : 0;
}

cudaError_t step_plan_create(const StepPhaseIn* in, int n, int n_heads, int n_kv, int64_t max_seq,
                             int device, StepPlan** out, const StepTp* tp) {
  *out = nullptr;
  if (n <= 0 || n_kv <= 0 || n_heads % n_kv) return cudaErrorInvalidValue;
  const bool tpm = tp && tp->world > 1;
  if (tpm && (tp->world > kMaxTp || tp->rank < 0 || tp->rank >= tp->world || tp->hidden <= 0 || tp->hidden % 8))
    return cudaErrorInvalidValue;
  const int G = n_heads / n_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return cudaErrorInvalidValue;
  // each attention phase is followed by its merge phase
  int nph = n;
  for (int i = 0; i < n; ++i) nph += in[i].kind == 1 ? 1 : 0;
  std::vector<PhaseDev> ph((size_t)nph);
  int need = 0, Umax = 0, redmax = 0;
  uint32_t mask = 0;
  for (int i = 0, o = 0; i < n; ++i, ++o) {
    std::memset(&ph[o], 0, sizeof(PhaseDev));
    if (in[i].kind == 0) {
      int slot = 0;
      if (!plan_gemv(in[i].g, &ph[o], &slot)) return cudaErrorInvalidValue;
      ph[o].cand = in[i].cand && in[i].g.nseg == 1 && !tpm ? 1 : 0;
      if (tpm) {
        ph[o].x_sum = in[i].x_sum;
        ph[o].xchg = in[i].xchg;
        if (in[i].xchg && (in[i].g.nseg != 1 || in[i].g.seg[0].mode != kStore)) return cudaErrorInvalidValue;
        if (in[i].x_sum && in[i].g.K != tp->hidden) return cudaErrorInvalidValue;
      } else if (in[i].x_sum || in[i].xchg) {
        return cudaErrorInvalidValue;
      }
      need = std::max(need, slot);
      Umax = std::max(Umax, ph[o].U);
      redmax = std::max(redmax, ph[o].red_floats);
      for (int k = 0; k < in[i].g.nseg; ++k) mask |= type_mask(in[i].g.seg[k].type);
    } else {
      ph[o].kind = 1;
      ph[o].a = in[i].a;
      ++o;
      std::memset(&ph[o], 0, sizeof(PhaseDev));
      ph[o].kind = 2;
      ph[o].a = in[i].a;
    }
  }
  StepPlan* P = new StepPlan();
  P->grid = sms_of(device);
  P->n_kv = n_kv;
  P->G = G;
  P->splits = P->grid / n_kv;
  {  // at most as many splits as let the merge phase stage its (output, split)
     // items in one pass over the consumers: a second pass is another L2 round
     // trip on the critical path (17 instead of 18 splits for the 4B shape)
    const int slice = (n_kv * G * 128 + P->grid - 1) / P->grid;
    P->splits = std::max(1, std::min(P->splits, kNC / std::max(1, slice)));
  }
  P->max_seq = max_seq;
  P->mask = mask;
  P->nph = nph;
  if (P->splits < 1) {
    delete P;
    return cudaErrorInvalidValue;
  }
  Geometry& g = P->geo;
  g.ucon_off = kPhaseBufOff + (int)((2 * sizeof(PhaseDev) + 127) & ~size_t(127));
  g.lim_off = g.ucon_off + ((20 * Umax + 127) & ~127);
  g.red_off = g.lim_off + 192 * Umax;
  int end = g.red_off + ((2 * redmax * 4 + 127) & ~127);
  const int attn_scratch = (G * 128 + kAttnWarps * G * 128 + 2 * kAttnWarps * G + 256) * 4;
  end = std::max(end, g.lim_off + ((attn_scratch + 127) & ~127));
  // the merge phase stages (output, split) triples of its slice of outputs
  const int merge_scratch = ((n_kv * G * 128 + P->grid - 1) / P->grid) * P->splits * 12;
  end = std::max(end, g.lim_off + ((merge_scratch + 127) & ~127));
  g.ring_off = (end + 127) & ~127;
  const int stage_bytes = std::max(need, 2 * 16 * 512);  // an attention tile holds 16 positions at least
  g.stage_bytes = stage_bytes;
  g.stages = std::min(kMaxStages, (kSmemMax - g.ring_off) / stage_bytes);
  if (g.stages < 2) {
    delete P;
    return cudaErrorInvalidValue;
  }
  g.attn_half = (stage_bytes / 2) & ~15;
  g.tile_pos = g.attn_half / 512;
  g.smem = g.ring_off + g.stages * stage_bytes;
  // second pass: a segment whose rows of one CTA fit one slot takes one
  // stage; a phase whose partials fit both buffers reduces once at its end
  for (int i = 0; i < nph; ++i) {
    PhaseDev& d = ph[i];
    if (d.kind != 0) continue;
    int total = 0;
    for (int l = 0; l < d.nls; ++l)
      total += ((d.ls[l].rows + P->grid - 1) / P->grid) * (d.ls[l].pair + 1) * (d.U | 1);
    d.deferred = total <= 2 * d.red_floats ? 1 : 0;
    if (!d.deferred) continue;  // chunked: the buffers are sized for the planned stages
    for (int l = 0; l < d.nls; ++l) {
      SLSeg& L = d.ls[l];
      const int64_t rb = d.seg[L.first].row_bytes;
      const int per_cta = (L.rows + P->grid - 1) / P->grid;
      const int64_t one = ((int64_t)per_cta * rb + 32 + 127) & ~int64_t(127);
      if (per_cta > L.m && one * (L.pair + 1) <= stage_bytes && (!L.pair || one <= d.half_bytes))
        L.m = per_cta;
    }
  }
  if (!fits(mask, G, g.smem, tpm)) {
    delete P;
    return cudaErrorInvalidValue;
  }
  if (tpm) {
    // exchange k of a launch: inbox slot k & 1; the residual before it is the
    // phase's own input (the embedding) for k = 0, else buffer (k - 1) & 1,
    // and the residual after it goes to buffer k & 1
    P->tp = *tp;
    int k = 0, last = -1;
    for (int i = 0, o = 0; i < n; ++i, ++o) {
      PhaseDev& d = ph[o];
      if (in[i].kind != 0) {
        ++o;
        continue;
      }
      if (d.x_sum) {
        if (last < 0) {
          delete P;
          return cudaErrorInvalidValue;  // no exchange before it
        }
        d.x_xk = last;
      }
      if (d.xchg) {
        d.xchg_k = k;
        last = k++;
      }
    }
    P->n_xchg = k;
    int max_xk = -1;  // the last exchange whose sum a later phase reads
    for (const PhaseDev& d : ph)
      if (d.kind == 0 && d.x_sum) max_xk = std::max(max_xk, d.x_xk);
    if (k == 0 || !ph[nph - 1].xchg) {  // the last phase gathers the output to every rank
      delete P;
      return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaMalloc(&P->arena, arena_bytes(P->tp));
    if (e == cudaSuccess) e = cudaMemset(P->arena, 0, arena_bytes(P->tp));
    if (e == cudaSuccess)  // inbox words: tag 0xFFFFFFFF, no exchange's
      e = cudaMemset(P->arena + inbox_off(P->tp, 0), 0xFF, inbox_off(P->tp, 2) - inbox_off(P->tp, 0));
    if (e != cudaSuccess) {
      if (P->arena) cudaFree(P->arena);
      delete P;
      return e;
    }
    for (int i = 0, o = 0; i < n; ++i, ++o) {
      PhaseDev& d = ph[o];
      if (in[i].kind != 0) {
        ++o;
        continue;
      }
      if (d.x_sum) {
        const int x = d.x_xk;
        d.inbox = reinterpret_cast<const uint64_t*>(P->arena + inbox_off(P->tp, x & 1));
        d.xr_prev = x == 0 ? in[i].g.x : reinterpret_cast<const float*>(P->arena + xr_off(P->tp, (x - 1) & 1));
        d.xr_next = x < max_xk ? reinterpret_cast<float*>(P->arena + xr_off(P->tp, x & 1)) : nullptr;
      }
    }
    P->table = ph;
    P->bound = false;
    *out = P;
    return cudaSuccess;
  }
  cudaError_t e = cudaMalloc(&P->dev, sizeof(PhaseDev) * (size_t)nph);
  if (e == cudaSuccess)
    e = cudaMemcpy(P->dev, ph.data(), sizeof(PhaseDev) * (size_t)nph, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (P->dev) cudaFree(P->dev);
    delete P;
    return e;
  }
  *out = P;
  return cudaSuccess;
}

void step_plan_free(StepPlan* p) {
  if (!p) return;
  if (p->dev) cudaFree(p->dev);
  if (p->arena) cudaFree(p->arena);
  delete p;
}

void* step_plan_tp_arena(const StepPlan* p) { return p ? p->arena : nullptr; }

cudaError_t step_plan_tp_bind(StepPlan* p, void* const* arenas, float* const* outputs) {
  if (!p || p->bound || !p->arena) return cudaErrorInvalidValue;
  const StepTp& t = p->tp;
  for (int r = 0; r < t.world; ++r) {
    if (!arenas[r] || !outputs[r]) return cudaErrorInvalidValue;
    p->xctr_rank[r] = static_cast<unsigned long long*>(arenas[r]);
  }
  for (PhaseDev& d : p->table) {
    if (d.kind != 0 || !d.xchg) continue;
    for (int r = 0; r < t.world; ++r)
      d.xdst[r] = d.xchg == 1 ? static_cast<void*>(reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(arenas[r]) +
                                                                               inbox_off(t, d.xchg_k & 1)) +
                                                   (size_t)t.rank * t.hidden)
                              : static_cast<void*>(outputs[r] + t.gather_offset);
  }
  cudaError_t e = cudaMalloc(&p->dev, sizeof(PhaseDev) * p->table.size());
  if (e == cudaSuccess)
    e = cudaMemcpy(p->dev, p->table.data(), sizeof(PhaseDev) * p->table.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (p->dev) cudaFree(p->dev);
    p->dev = nullptr;
    return e;
  }
  p->bound = true;
  return cudaSuccess;
}

int step_plan_splits(const StepPlan* p) { return p ? p->splits : 0; }
int step_plan_grid(const StepPlan* p) { return p ? p->grid : 0; }

cudaError_t step_launch(const StepPlan* plan, DecodeState* st, const float* rope, float eps,
                        float* part, uint32_t* ctr, int32_t* err, const LogitCands* cands, cudaStream_t s) {
  if (!plan->bound) return cudaErrorInvalidValue;
  StepParams p{};
  p.ph = plan->dev;
  p.nph = plan->nph;
  p.tp_world = plan->tp.world;
  p.n_xchg = plan->n_xchg;
  if (plan->tp.world > 1) {
    p.xctr = reinterpret_cast<unsigned long long*>(plan->arena);
    p.launches = reinterpret_cast<unsigned long long*>(plan->arena + kLaunchOff);
    p.tp_rank = plan->tp.rank;
    for (int r = 0; r < plan->tp.world; ++r) p.xctr_rank[r] = plan->xctr_rank[r];
  }
  p.st = st;
  if (cands && cands->val && cands->ctas == plan->grid) p.cands = *cands;
  p.rope = rope;
  p.eps = eps;
  p.n_kv = plan->n_kv;
  p.splits = plan->splits;
  p.max_seq = plan->max_seq;
  p.part = part;
  p.ctr = ctr;
  p.err = err;
  p.stages = plan->geo.stages;
  p.stage_bytes = plan->geo.stage_bytes;
  p.tile_pos = plan->geo.tile_pos;
  p.attn_half = plan->geo.attn_half;
  p.ucon_off = plan->geo.ucon_off;
  p.lim_off = plan->geo.lim_off;
  p.red_off = plan->geo.red_off;
  p.ring_off = plan->geo.ring_off;
  const uint32_t m = plan->mask;
  if (plan->tp.world > 1) {
    if (m == kMQ80) return launch_tm<kMQ80, true>(p, plan->G, plan->grid, plan->geo.smem, s);
    return launch_tm<kMQ4K | kMQ6K | kMQ80, true>(p, plan->G, plan->grid, plan->geo.smem, s);
  }
  if ((m & ~(kMQ4K | kMQ6K)) == 0) return launch_tm<kMQ4K | kMQ6K, false>(p, plan->G, plan->grid, plan->geo.smem, s);
  if (m == kMQ80) return launch_tm<kMQ80, false>(p, plan->G, plan->grid, plan->geo.smem, s);
  return launch_tm<kMQ4K | kMQ6K | kMQ80, false>(p, plan->G, plan->grid, plan->geo.smem, s);
}

}  // namespace rpgc
