// k_sample.cu -- greedy / sampled token choice on the device (one block).
//
// Reference: ArgMax (src/kernels.h:42-52), CounterUniform
// (src/sampler.cc:16-34), FilterToProbs + SampleToken (src/sampler.cc:36-112):
//   temperature -> top-k (keep >= k-th largest, 1 < k < n) -> softmax (double
//   sum) -> top-p (ascending cumulative sum, zero while cum <= 1-p, keep the
//   largest) -> renormalise -> first index whose cumulative sum exceeds u.
//
// Device formulation.  The k-th largest value is a 4-pass radix select over
// order-preserving float keys.  The top-p cut is a 4-pass radix search over
// the probability bits whose bucket masses are exact 2^-62 fixed-point sums,
// which locates the first element (ascending value, ties by index) whose
// running sum exceeds 1-p without sorting.  The inverse CDF uses the same
// exact fixed-point prefix sums in index order.  Softmax/renormalisation sums
// are double, reduced in a fixed order (deterministic).  When top-k is active
// its survivors are compacted (index order kept) and the later passes run on
// them only.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace rpgc {
namespace {

constexpr int NT = 1024;
constexpr int kCap = 4864;  // compacted survivors held in shared memory (>= 148 CTAs x kCandK candidates)
constexpr double kFix = 4611686018427387904.0;  // 2^62

struct Smem {
  uint32_t cnt[32][256];
  unsigned long long msum[32][256];
  int cidx[kCap];
  float cval[kCap];
  double dred[NT];
  unsigned long long ured[NT];
  int ired[NT];
  float fred[32];
  int ibest[32];
  unsigned long long bcast_u[4];
  double bcast_d[2];
  int bcast_i[8];
  float bcast_f[4];
};

__device__ __forceinline__ uint32_t fkey(float f) {  // order-preserving
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unfkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
__device__ float counter_uniform(uint64_t seed, uint64_t counter) {
  const uint32_t bits = (uint32_t)(splitmix64(seed + 0x9E3779B97F4A7C15ull * counter) >> 40);
  return (float)bits * (1.0f / 16777216.0f);
}

// ---- block reductions (1024 threads) ------------------------------------
// Fixed pairing order: element i takes i + st for st = NT/2, ..., 1 (the
// same additions in the same order whatever the layout below).  The first
// three levels run in shared memory; warp 0 does the rest in registers (its
// lane l holds elements l + 32k, k < 4, then shuffles down for st < 32).
__device__ double block_sum_d(Smem& S, double v) {
  static_assert(NT == 1024, "three shared-memory levels leave 128 elements");
  S.dred[threadIdx.x] = v;
  __syncthreads();
  for (int st = NT / 2; st >= 128; st >>= 1) {
    if (threadIdx.x < st) S.dred[threadIdx.x] += S.dred[threadIdx.x + st];
    __syncthreads();
  }
  if (threadIdx.x < 32) {
    const int l = threadIdx.x;
    double a0 = S.dred[l], a1 = S.dred[l + 32], a2 = S.dred[l + 64], a3 = S.dred[l + 96];
    a0 += a2;  // st = 64
    a1 += a3;
    a0 += a1;  // st = 32
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a0 += __shfl_down_sync(0xffffffffu, a0, o);
    if (l == 0) S.bcast_d[0] = a0;
  }
  __syncthreads();
  const double r = S.bcast_d[0];
  __syncthreads();
  return r;
}
__device__ float block_max_f(Smem& S, float v) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) S.fred[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = S.fred[threadIdx.x];
    w = warp_max(w);
    if (threadIdx.x == 0) S.bcast_f[0] = w;
  }
  __syncthreads();
  const float r = S.bcast_f[0];
  __syncthreads();
  return r;
}
// (value, index): larger value wins, ties -> smaller index.  NaN never wins.
__device__ int block_argmax(Smem& S, float v, int i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    S.fred[threadIdx.x >> 5] = v;
    S.ibest[threadIdx.x >> 5] = i;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    v = S.fred[threadIdx.x];
    i = S.ibest[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
      }
    }
    if (threadIdx.x == 0) S.bcast_i[0] = i;
  }
  __syncthreads();
  const int r = S.bcast_i[0];
  __syncthreads();
  return r;
}
// exclusive prefix over threads (integers are exact, order irrelevant): a
// shuffle scan in each warp, then one over the 32 warp totals
template <typename T>
__device__ T block_excl_scan(T* buf, T v, T* total) {
  static_assert(NT == 1024, "32 warps");
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) buf[w] = x;
  __syncthreads();
  if (w == 0) {
    T t = buf[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    buf[32 + lane] = t;
  }
  __syncthreads();
  const T off = w ? buf[32 + w - 1] : T(0);
  *total = buf[63];
  __syncthreads();
  return off + x - v;
}

__device__ void clear_hist(Smem& S, bool sums) {
  for (int i = threadIdx.x; i < 32 * 256; i += NT) {
    (&S.cnt[0][0])[i] = 0;
    if (sums) (&S.msum[0][0])[i] = 0;
  }
  __syncthreads();
}

// Candidate view: element j of [0, m).
struct View {
  const float* logits;
  float invT;
  bool scaled;
  bool compact;
  const int* idx;
  const float* val;
  float kth;     // top-k floor (-inf when off)
  float mx;      // softmax max
  float inv;     // softmax 1/sum
  int m;
};
__device__ __forceinline__ float v_s(const View& v, int j) {
  float s = v.compact ? v.val[j] : (v.scaled ? v.logits[j] * v.invT : v.logits[j]);
  return s < v.kth ? -INFINITY : s;
}
__device__ __forceinline__ int v_i(const View& v, int j) { return v.compact ? v.idx[j] : j; }
__device__ __forceinline__ float v_p(const View& v, int j) {  // softmax output (float)
  return expf(v_s(v, j) - v.mx) * v.inv;
}

// k-th largest value of V's elements [0, m) (4-pass radix select over the
// order-preserving keys; the count of equal values decides, as nth_element's
// "keep >= k-th" does).
__device__ float kth_largest(Smem& S, const View& V, int m, int k) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  int krem = k;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    clear_hist(S, false);
    const int w = tid >> 5;
    for (int j = tid; j < m; j += NT) {
      const uint32_t kk = fkey(v_s(V, j));
      if ((kk & pmask) == prefix) atomicAdd(&S.cnt[w][(kk >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid < 256) {
      uint32_t c = 0;
      for (int ww = 0; ww < 32; ++ww) c += S.cnt[ww][tid];
      S.cnt[0][tid] = c;
    }
    __syncthreads();
    if (tid < 32) {
      // the highest bin b >= 1 whose count from b up reaches krem (0 if none)
      // and the count above it: lane l holds bins 8l .. 8l+7
      int c[8], tl = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = (int)S.cnt[0][8 * tid + j];
        tl += c[j];
      }
      int sfx = tl;  // inclusive suffix over lanes l..31
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_down_sync(0xffffffffu, sfx, o);
        if (tid + o < 32) sfx += y;
      }
      int run = sfx - tl, best = -1, best_above = 0;  // run: count of bins above the lane's
#pragma unroll
      for (int j = 7; j >= 0; --j) {
        const int b = 8 * tid + j;
        if (b >= 1 && best < 0 && run + c[j] >= krem) {
          best = b;
          best_above = run;
        }
        run += c[j];
      }
      // the highest lane with a qualifying bin holds b*
      const unsigned q = __ballot_sync(0xffffffffu, best >= 0);
      const int src = q ? 31 - __clz((int)q) : 0;
      const int b = q ? __shfl_sync(0xffffffffu, best, src) : 0;
      const int above = q ? __shfl_sync(0xffffffffu, best_above, src) : __shfl_sync(0xffffffffu, sfx - c[0], 0);
      if (tid == 0) {
        S.bcast_i[1] = b;
        S.bcast_i[2] = krem - above;
      }
    }
    __syncthreads();
    prefix |= (uint32_t)S.bcast_i[1] << shift;
    pmask |= 255u << shift;
    krem = S.bcast_i[2];
    __syncthreads();
  }
  return unfkey(prefix);
}

// The full vocabulary with temperature and top-k applied: survivors
// compacted (index order kept) when they fit shared memory.
__device__ View view_full(Smem& S, const float* logits, int n, float T, int top_k) {
  const int tid = threadIdx.x;
  View V;
  V.logits = logits;
  V.scaled = (T != 1.0f);
  V.invT = 1.0f / T;
  V.compact = false;
  V.idx = S.cidx;
  V.val = S.cval;
  V.kth = -INFINITY;
  V.m = n;
  if (top_k > 1 && top_k < n) {
    V.kth = kth_largest(S, V, n, top_k);
    // compact survivors in index order when they fit: warp w owns a
    // contiguous index range, read 32 consecutive logits per round
    // (coalesced); ballots give each survivor its slot.
    const int w = tid >> 5, lane = tid & 31;
    const int R = ((n + 32 * 32 - 1) / (32 * 32)) * 32;  // range length per warp
    const int w0 = w * R, w1 = min(n, w0 + R);
    int mine = 0;
    for (int j = w0 + lane; j - lane < w1; j += 32) {
      const bool keep = j < w1 && v_s(V, j) != -INFINITY;
      mine += __popc(__ballot_sync(0xffffffffu, keep));
    }
    if (lane == 0) S.ired[w] = mine;
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      for (int ww = 0; ww < 32; ++ww) {
        const int c = S.ired[ww];
        S.ired[ww] = acc;
        acc += c;
      }
      S.bcast_i[3] = acc;
    }
    __syncthreads();
    const int total = S.bcast_i[3];
    if (total <= kCap) {
      int o = S.ired[w];
      for (int j = w0 + lane; j - lane < w1; j += 32) {
        const float sv = j < w1 ? v_s(V, j) : -INFINITY;
        const bool keep = sv != -INFINITY;
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (keep) {
          const int at = o + __popc(bal & ((1u << lane) - 1u));
          S.cidx[at] = j;
          S.cval[at] = sv;
        }
        o += __popc(bal);
      }
      __syncthreads();
      V.compact = true;
      V.m = total;
      V.kth = -INFINITY;  // survivors only
    }
  }
  return V;
}

// softmax -> top-p -> renormalise -> inverse CDF over the view's elements.
__device__ int sample_view(Smem& S, View V, float top_p, float u) {
  const int tid = threadIdx.x;
  const int m = V.m;
  const int C = (m + NT - 1) / NT, j0 = tid * C, j1 = min(m, j0 + C);
  // ---------------- softmax
  float lmax = -INFINITY;
  for (int j = j0; j < j1; ++j) lmax = fmaxf(lmax, v_s(V, j));
  V.mx = block_max_f(S, lmax);
  V.inv = 1.0f;
  double le = 0.0;
  for (int j = j0; j < j1; ++j) le += (double)expf(v_s(V, j) - V.mx);
  V.inv = (float)(1.0 / block_sum_d(S, le));
  // ---------------- top-p: first ascending element whose running mass > 1-p
  const bool do_p = top_p > 0.0f && top_p < 1.0f;
  uint32_t vkey = 0;      // crossing value (probability bits)
  long long n_zero_ties = 0;
  bool all_zero = false;
  if (do_p) {
    const double thr = 1.0 - (double)top_p;
    const unsigned long long thr_fp = (unsigned long long)(thr * kFix);
    unsigned long long below = 0;  // mass of elements with key < prefix range
    uint32_t prefix = 0, pmask = 0;
    bool crossed = true;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      clear_hist(S, true);
      const int w = tid >> 5;
      for (int j = j0; j < j1; ++j) {
        const float p = v_p(V, j);
        const uint32_t k = __float_as_uint(p);
        if ((k & pmask) == prefix) {
          const uint32_t b = (k >> shift) & 255u;
          atomicAdd(&S.cnt[w][b], 1u);
          atomicAdd(&S.msum[w][b], (unsigned long long)((double)p * kFix));
        }
      }
      __syncthreads();
      if (tid < 256) {
        uint32_t c = 0;
        unsigned long long s = 0;
        for (int ww = 0; ww < 32; ++ww) {
          c += S.cnt[ww][tid];
          s += S.msum[ww][tid];
        }
        S.cnt[0][tid] = c;
        S.msum[0][tid] = s;
      }
      __syncthreads();
      if (tid < 32) {
        // the lowest bin b whose mass from below up to and including it
        // exceeds thr_fp (256 if none): lane l holds bins 8l .. 8l+7
        unsigned long long m8[8], tl = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          m8[j] = S.msum[0][8 * tid + j];
          tl += m8[j];
        }
        unsigned long long pre = tl;  // inclusive prefix over lanes 0..l
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned long long y = __shfl_up_sync(0xffffffffu, pre, o);
          if (tid >= o) pre += y;
        }
        unsigned long long cum = below + (pre - tl);
        int best = 256;
        unsigned long long best_cum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (best == 256 && cum + m8[j] > thr_fp) {
            best = 8 * tid + j;
            best_cum = cum;
          }
          cum += m8[j];
        }
        const unsigned q = __ballot_sync(0xffffffffu, best < 256);
        const int src = q ? __ffs((int)q) - 1 : 0;
        const int b = q ? __shfl_sync(0xffffffffu, best, src) : 256;
        const unsigned long long bc = __shfl_sync(0xffffffffu, best_cum, src);
        const unsigned long long all = __shfl_sync(0xffffffffu, cum, 31);
        if (tid == 0) {
          S.bcast_i[1] = b;
          S.bcast_u[0] = q ? bc : all;
          S.bcast_i[3] = (b < 256) ? (int)S.cnt[0][b] : 0;
        }
      }
      __syncthreads();
      const int b = S.bcast_i[1];
      if (b == 256) {  // never exceeds: every element is zeroed
        crossed = false;
        __syncthreads();
        break;
      }
      prefix |= (uint32_t)b << shift;
      pmask |= 255u << shift;
      below = S.bcast_u[0];
      __syncthreads();
    }
    if (crossed) {
      vkey = prefix;
      const unsigned long long vfp = (unsigned long long)((double)__uint_as_float(vkey) * kFix);
      // ties: the j-th (index order) equal element has running mass below+(j+1)*v
      n_zero_ties = (vfp > 0 && thr_fp >= below) ? (long long)((thr_fp - below) / vfp) : 0;
    } else {
      all_zero = true;
    }
  }
  // tie ranks of the crossing value, per thread chunk
  int my_ties = 0;
  if (do_p && !all_zero)
    for (int j = j0; j < j1; ++j) my_ties += (__float_as_uint(v_p(V, j)) == vkey);
  int tot_ties;
  const int tie_base = block_excl_scan<int>(S.ired, my_ties, &tot_ties);
  // last index of the maximum (the largest element in ascending order)
  int keep_last = -1;
  if (do_p && all_zero) {
    // largest value, ties -> largest index: argmax over (value, -index)
    float bv = -INFINITY;
    int bi = -1;
    for (int j = j0; j < j1; ++j) {
      const float p = v_p(V, j);
      if (p > bv || (p == bv && v_i(V, j) > bi)) {
        bv = p;
        bi = v_i(V, j);
      }
    }
    const int neg = block_argmax(S, bv, bi >= 0 ? -bi : 0x7fffffff);
    keep_last = -neg;
  }
  // final probability of element j (after top-p and before renormalisation)
  auto q_raw = [&](int j, int tie_rank) -> float {
    const float p = v_p(V, j);
    if (!do_p) return p;
    if (all_zero) return v_i(V, j) == keep_last ? 1.0f : 0.0f;
    const uint32_t k = __float_as_uint(p);
    if (k < vkey) return 0.0f;
    if (k == vkey && tie_rank < n_zero_ties) return 0.0f;
    return p;
  };
  float inv2 = 1.0f;
  if (do_p) {
    double ls = 0.0;
    int r = tie_base;
    for (int j = j0; j < j1; ++j) {
      const bool tie = !all_zero && __float_as_uint(v_p(V, j)) == vkey;
      ls += (double)q_raw(j, r);
      r += tie;
    }
    const double tot = block_sum_d(S, ls);
    if (tot > 0.0) inv2 = (float)(1.0 / tot);
  }
  // ---------------- inverse CDF in index order (exact fixed-point prefix)
  unsigned long long mine = 0;
  {
    int r = tie_base;
    for (int j = j0; j < j1; ++j) {
      const bool tie = do_p && !all_zero && __float_as_uint(v_p(V, j)) == vkey;
      const float q = do_p ? q_raw(j, r) * inv2 : q_raw(j, r);
      mine += (unsigned long long)((double)q * kFix);
      r += tie;
    }
  }
  unsigned long long totm;
  const unsigned long long before = block_excl_scan<unsigned long long>(S.ured, mine, &totm);
  const unsigned long long ufp = (unsigned long long)((double)u * kFix);
  if (tid == 0) S.bcast_i[4] = 0x7fffffff;
  __syncthreads();
  if (before <= ufp && ufp < before + mine) {  // the crossing lies in this chunk
    unsigned long long cum = before;
    int r = tie_base;
    for (int j = j0; j < j1; ++j) {
      const bool tie = do_p && !all_zero && __float_as_uint(v_p(V, j)) == vkey;
      const float q = do_p ? q_raw(j, r) * inv2 : q_raw(j, r);
      cum += (unsigned long long)((double)q * kFix);
      r += tie;
      if (cum > ufp) {
        S.bcast_i[4] = v_i(V, j);
        break;
      }
    }
  }
  __syncthreads();
  int tok = S.bcast_i[4];
  __syncthreads();
  if (tok == 0x7fffffff) {  // u beyond the total mass: most probable token
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    int r = tie_base;
    for (int j = j0; j < j1; ++j) {
      const bool tie = do_p && !all_zero && __float_as_uint(v_p(V, j)) == vkey;
      const float q = do_p ? q_raw(j, r) * inv2 : q_raw(j, r);
      r += tie;
      if (q > bv || (q == bv && v_i(V, j) < bi)) {
        bv = q;
        bi = v_i(V, j);
      }
    }
    tok = block_argmax(S, bv, bi);
  }
  return tok;
}

__device__ int sample_probs(Smem& S, const float* logits, int n, float T, int top_k, float top_p, float u) {
  return sample_view(S, view_full(S, logits, n, T, top_k), top_p, u);
}

// The top-k survivors from the decode step's candidates (LogitCands): the
// valid entries of every CTA's list (index order within a CTA, CTAs in
// vocabulary order, so index order overall), the k-th largest of their
// scaled values, and the survivors >= it.  Returns false -- the caller then
// takes the full vocabulary -- when a CTA whose list is full has its
// smallest listed value >= the k-th: it may hold more such elements than it
// listed (ties), which only the full sweep sees.
__device__ bool view_cands(Smem& S, const LogitCands& c, float T, int top_k, View* out) {
  const int tid = threadIdx.x;
  const float invT = 1.0f / T;
  const bool scaled = (T != 1.0f);
  const int slots = c.ctas * kCandK;  // <= kCap (checked by the caller)
  constexpr int kPer = (kCap + NT - 1) / NT;
  // 1. the valid entries, compacted in slot order (each thread's chunk read, then written)
  const int C = (slots + NT - 1) / NT, s0 = tid * C, s1 = min(slots, s0 + C);
  float vv[kPer];
  int vi[kPer];
  int nv = 0;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int sl = s0 + q;
    vi[q] = -1;
    vv[q] = 0.0f;
    if (sl < s1) {
      const int i = c.idx[sl];
      if (i >= 0) {
        const float raw = c.val[sl];
        vv[q] = scaled ? raw * invT : raw;
        vi[q] = i;
        ++nv;
      }
    }
  }
  int m;
  const int base = block_excl_scan<int>(S.ired, nv, &m);
  {
    int o = base;
#pragma unroll
    for (int q = 0; q < kPer; ++q)
      if (vi[q] >= 0) {
        S.cidx[o] = vi[q];
        S.cval[o] = vv[q];
        ++o;
      }
  }
  __syncthreads();
  View V;
  V.logits = nullptr;
  V.scaled = false;
  V.invT = 1.0f;
  V.compact = true;
  V.idx = S.cidx;
  V.val = S.cval;
  V.kth = -INFINITY;
  V.m = m;
  if (top_k >= m) return false;  // every list short, so m is the vocabulary: no filtering to do here
  const float kth = kth_largest(S, V, m, top_k);
  // 2. a full list whose smallest value reaches the k-th: possibly incomplete
  bool risky = false;
  if (tid < c.ctas && c.idx[tid * kCandK + kCandK - 1] >= 0) {
    float lo = INFINITY;
    for (int q = 0; q < kCandK; ++q) {
      const float raw = c.val[tid * kCandK + q];
      lo = fminf(lo, scaled ? raw * invT : raw);
    }
    risky = lo >= kth;
  }
  if (__syncthreads_or(risky)) return false;
  // 3. survivors >= k-th, order kept
  const int C2 = (m + NT - 1) / NT, j0 = tid * C2, j1 = min(m, j0 + C2);
  float sv[kPer];
  int si[kPer];
  int ns = 0;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int j = j0 + q;
    si[q] = -1;
    sv[q] = 0.0f;
    if (j < j1 && S.cval[j] >= kth) {
      sv[q] = S.cval[j];
      si[q] = S.cidx[j];
      ++ns;
    }
  }
  int total;
  const int b2 = block_excl_scan<int>(S.ired, ns, &total);  // its barriers order the reads before the writes
  {
    int o = b2;
#pragma unroll
    for (int q = 0; q < kPer; ++q)
      if (si[q] >= 0) {
        S.cidx[o] = si[q];
        S.cval[o] = sv[q];
        ++o;
      }
  }
  __syncthreads();
  V.m = total;
  *out = V;
  return true;
}

__global__ void __launch_bounds__(NT) sample_kernel(const SampleArgs a) {
  extern __shared__ __align__(16) uint8_t raw[];
  Smem& S = *reinterpret_cast<Smem*>(raw);
  grid_dep_wait();
  // batched decode: block b is session b (its logits row, state, outputs and
  // embedding row); otherwise the single-session fields
  const int b = (int)blockIdx.x;
  DecodeState* st = a.states ? a.states[b] : a.state;
  const float* logits = a.logits + (int64_t)b * a.n;
  int32_t* out_ids = a.states ? a.out_ids_b[b] : a.out_ids;
  int32_t* n_out = a.states ? a.n_out_b[b] : a.n_out;
  float* xrow = a.x ? a.x + (int64_t)b * a.hidden : nullptr;
  float T = a.temperature, top_p = a.top_p, u = a.u;
  int top_k = a.top_k;
  int pos = 0;
  if (st) {
    const int done = st->done;
    __syncthreads();
    if (done) {
      if (threadIdx.x == 0) st->active = 0;
      return;
    }
    T = st->temperature;
    top_k = st->top_k;
    top_p = st->top_p;
    pos = st->start_pos + st->n_gen;  // where the picked token will be written
    u = counter_uniform(st->seed, (uint64_t)pos);
  }
  const int n = (int)a.n;
  // the step kernel's candidates of these logits, when it left the kind the
  // options need and no CTA saw a NaN (max_idx -2): then the sweep of the
  // whole vocabulary is skipped
  const LogitCands& cd = a.cands;
  int cmode = (st && cd.max_idx && cd.ctas > 0 && cd.ctas <= NT && cd.ctas * kCandK <= kCap) ? st->cand_ok : 0;
  if (__syncthreads_or(cmode > 0 && threadIdx.x < cd.ctas && cd.max_idx[threadIdx.x] == -2)) cmode = 0;
  int tok = -1;
  if (!(T > 0.0f)) {  // greedy: first index of the maximum
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    if (cmode >= 1) {  // the CTAs' maxima, in vocabulary order
      if (threadIdx.x < cd.ctas && cd.max_idx[threadIdx.x] >= 0) {
        bv = cd.max_val[threadIdx.x];
        bi = cd.max_idx[threadIdx.x];
      }
    } else {
      for (int j = threadIdx.x; j < n; j += NT) {  // coalesced sweep
        const float v = logits[j];
        if (v > bv) {  // a thread's indices increase, so strict > keeps the first
          bv = v;
          bi = j;
        }
      }
    }
    tok = block_argmax(S, bv, bi);
    if (tok == 0x7fffffff) tok = 0;
  } else {
    View V;
    if (cmode == 2 && top_k > 1 && top_k <= kCandK && top_k < n && view_cands(S, cd, T, top_k, &V))
      tok = sample_view(S, V, top_p, u);
    else
      tok = sample_probs(S, logits, n, T, top_k, top_p, u);
  }
  if (st && xrow) {  // the decode step continues with this token's embedding row
    const uint8_t* row = a.embd + (int64_t)tok * a.embd_row_bytes;
    for (int e = threadIdx.x; e < a.hidden; e += NT) xrow[e] = deq_elem(a.embd_type, row, e);
  }
  if (threadIdx.x == 0) {
    if (st) {
      st->pos = pos;
      st->token = tok;
      out_ids[st->n_gen] = tok;
      st->n_gen += 1;
      st->active = 1;
      bool stop = false;
      for (int i = 0; i < st->n_stop; ++i) stop |= (st->stop_ids[i] == tok);
      if (stop || st->n_gen >= st->max_tokens) st->done = 1;
      if (n_out) *n_out = st->n_gen;
    } else {
      *a.token_out = tok;
    }
  }
}

}  // namespace

cudaError_t sample_launch(const SampleArgs& a, cudaStream_t s) {
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(Smem));
    if (e != cudaSuccess) return e;
    configured = dev;
  }
  if (a.n <= 0 || a.n > 0x7ffffff0) return cudaErrorInvalidValue;
  if (a.states && (a.nbatch < 1 || !a.out_ids_b || !a.n_out_b)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.states ? (unsigned)a.nbatch : 1u);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = sizeof(Smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  const cudaError_t e_ = cudaLaunchKernelEx(&cfg, sample_kernel, a);
  if (e_ == cudaSuccess) count_launches(1);
  return e_;
}

}  // namespace rpgc
