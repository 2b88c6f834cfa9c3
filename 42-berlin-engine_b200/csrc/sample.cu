// sample.cu -- device sampling: the reference server's sampling step
// (worker.c:436-497 with sample_top_p, sampler_topp.c:113-158) and
// sample_temperature (sampler_temp.c:96-115).
//
// Top-p, per row, in the reference's order:
//   1. repetition penalty for every token of the history (prompt and
//      generated, repeats applied again): l > 0 ? l / p : l * p;
//   2. token 0 (UNK) blocked: l[0] = -1e9 (optional);
//   3. softmax at temperature t: m = max l, p_i = expf((l_i - m) / t) / sum;
//   4. probabilities in descending order (ties by index), the nucleus = the
//      shortest prefix whose running sum exceeds top_p;
//   5. r in [0, 1] (the caller's uniform draw: the reference uses
//      rand() / RAND_MAX) times the nucleus' mass; the token is the first
//      of the nucleus whose running sum exceeds it.
//
// Layout: one cluster of kCl CTAs per row; CTA c holds the c-th slice of the
// row in shared memory (logits, then probabilities), so every pass after
// the first load reads shared memory only.  Cluster-wide values (max, sum,
// histograms, counts) are exchanged through distributed shared memory and
// combined in a fixed order, so the result does not depend on scheduling.
//
// No sort is materialised.  The cut points of steps 4 and 5 are found by
// radix selection over the probabilities' bit patterns (positive floats
// order like unsigned integers) in three passes of 11, 11 and 9 bits, with
// the mass of every bin accumulated in 2^-50 fixed point (integer
// additions: exact in any order).  Both cuts run in the same three passes:
// the draw's target r * cum depends on the nucleus' mass cum, which lies
// within one tail probability of top_p, so the passes select for r * top_p
// beside top_p, and the result is checked against the exact r * cum
// afterwards; on a miss the draw is selected again.  A draw below the mass
// above the nucleus' cut needs no filter: the running sums there are those
// of the whole descending order.  Ties at a cut are taken in index order.
//
// The reference sums in float, in sorted order, so a draw within float
// rounding of a boundary can pick a token next to the reference's in that
// order.
#include <climits>
#include <cstdint>

#include <cooperative_groups.h>

#include "ec_internal.cuh"

namespace cg = cooperative_groups;

namespace ec {
namespace {

constexpr int kCl = 8;            // CTAs per row (portable cluster size)
constexpr int kThr = 512;         // threads per CTA
constexpr int kWarps = kThr / 32;
constexpr int kBins = 2048;       // histogram bins of the widest pass
constexpr int kMaxPortion = kBins / kCl;
constexpr double kFix = 1125899906842624.0;  // 2^50
constexpr int kMaxSlice = 40960;  // floats of one row per CTA (n <= 327680)
// two histograms (masses and counts), one per selection target
constexpr size_t kHistBytes = 2 * (size_t)kBins * (8 + 4);

struct SampleArgs {
  float* logits;
  int n;
  const int* history;
  const int* history_len;
  int history_stride;
  float temperature, top_p, penalty;
  int block0;
  const float* r;
  int* out;
};

typedef unsigned long long u64;

// Phase timestamps for performance work (build with -DEC_PHASE_TIMING):
// slot s of g_sample_ts gets %globaltimer when CTA 0's thread 0 passes it.
#ifdef EC_PHASE_TIMING
__device__ long long g_sample_ts[32];
#define SAMPLE_MARK(s)                                          \
  do {                                                          \
    if (blockIdx.x == 0 && threadIdx.x == 0) {                  \
      long long t_;                                             \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));   \
      g_sample_ts[s] = t_;                                      \
    }                                                           \
  } while (0)
#else
#define SAMPLE_MARK(s) \
  do {                 \
  } while (0)
#endif

__device__ __forceinline__ u64 fix(float p) { return (u64)((double)p * kFix); }

__device__ __forceinline__ void penalise_shared(float* a, float pen) {
  unsigned* p = reinterpret_cast<unsigned*>(a);
  unsigned old = *p, assumed;
  do {
    assumed = old;
    const float v = __uint_as_float(assumed);
    const float nv = v > 0.0f ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);
    old = atomicCAS(p, assumed, __float_as_uint(nv));
  } while (old != assumed);
}

// Block-wide reduction, combined in warp order (deterministic).
template <typename T, typename Op>
__device__ T block_reduce(T v, T* red, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T r = red[0];
  for (int w = 1; w < kWarps; w++) r = op(r, red[w]);
  return r;
}

// Per-CTA view of its slice of the row.
struct Slice {
  float* p;          // the slice (shared memory; 16-byte aligned)
  int c0, len;       // first row index of the slice, its length
  u64* hm;           // [2][kBins] bin masses, one histogram per target
  unsigned* hc;      // [2][kBins] bin counts
};

struct Exchange {    // static shared; the parts other CTAs read are marked
  float mx;                       // remote: this CTA's max
  double sum;                     // remote: its sum of exp values
  u64 tm;                         // remote: its fixed-point mass
  u64 pm[2][kMaxPortion];         // remote: its portion of the histograms
  unsigned pc[2][kMaxPortion];
  u64 port_m[2];                  // remote: the portion's totals
  unsigned port_c[2];
  u64 rs_m[2][kThr];              // local: reduce-scatter partial sums
  unsigned rs_c[2][kThr];
};

// Cut state of one selection target.
struct Cut {
  unsigned prefix;  // key bits fixed so far
  u64 above;        // mass strictly above the current bin
  unsigned cnt;     // elements in the final bin (after the last pass)
};

// Applies f(i, p) to every element of the slice, four at a time.
template <typename F>
__device__ __forceinline__ void for_slice(const Slice& s, F f) {
  const int n4 = s.len >> 2;
  const float4* p4 = reinterpret_cast<const float4*>(s.p);
  for (int i = threadIdx.x; i < n4; i += kThr) {
    const float4 v = p4[i];
    f(4 * i, v.x);
    f(4 * i + 1, v.y);
    f(4 * i + 2, v.z);
    f(4 * i + 3, v.w);
  }
  for (int i = 4 * n4 + threadIdx.x; i < s.len; i += kThr) f(i, s.p[i]);
}

// One radix pass over bits [shift, shift + log2(NB)) of the probabilities'
// bit patterns, for two selection targets at once (one histogram while both
// have the same prefix): for each target, the bin in which the running mass
// in descending order, among the elements matching its prefix under `mask`,
// first exceeds the target (the smallest non-empty bin if none does).
//   1. each CTA builds its own histograms (shared-memory atomics);
//   2. reduce-scatter: CTA c sums portion c (NB / kCl bins) of all CTAs'
//      histograms, and the portion's total;
//   3. every CTA walks the kCl portion totals from the top, then the bins of
//      the portion the target falls in, read from the CTA that owns it;
//      threads 0-255 walk for target 0, threads 256-511 for target 1.
// Two cluster barriers per pass; every buffer is rewritten only after the
// barrier that follows its last remote read.  FIRST: the slice holds exp
// values, which this pass divides by `sum` into probabilities.
template <int NB, bool FIRST>
__device__ void radix_pass(const Slice& s, Exchange& x, cg::cluster_group& cl, int shift,
                           unsigned mask, const u64* target, Cut* cut, float sum) {
  constexpr int PB = NB / kCl;  // bins per portion
  constexpr int G = kThr / PB;  // thread groups in the reduce-scatter
  static_assert(PB <= kMaxPortion && kThr % PB == 0 && kCl % G == 0, "portion shape");
  static_assert(kThr == 512 && PB <= 256, "one half-block walks each target");
  __shared__ u64 s_wt[kWarps];
  __shared__ unsigned s_wc[kWarps];
  __shared__ int s_first[kWarps], s_last[kWarps];
  __shared__ int s_q[2], s_cr[2];
  __shared__ u64 s_acc[2];
  __shared__ Cut s_cut[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rank = (int)cl.block_rank();
  const unsigned p0 = cut[0].prefix, p1 = cut[1].prefix;
  const bool two = p0 != p1;
  const int nh = two ? 2 : 1;
  for (int b = threadIdx.x; b < NB; b += kThr) {
    s.hm[b] = 0;
    s.hc[b] = 0;
    s.hm[kBins + b] = 0;
    s.hc[kBins + b] = 0;
  }
  __syncthreads();
  float* pw = s.p;
  for_slice(s, [&](int i, float v) {
    float p = v;
    if (FIRST) {
      p = __fdiv_rn(v, sum);
      pw[i] = p;
    }
    const unsigned k = __float_as_uint(p);
    const int b = (k >> shift) & (NB - 1);
    if ((k & mask) == p0) {
      atomicAdd(&s.hm[b], fix(p));
      atomicAdd(&s.hc[b], 1u);
    }
    if (two && (k & mask) == p1) {
      atomicAdd(&s.hm[kBins + b], fix(p));
      atomicAdd(&s.hc[kBins + b], 1u);
    }
  });
  cl.sync();
  {
    // group g sums ranks g*(kCl/G) .. (g+1)*(kCl/G)-1 for bin rank*PB + t
    const int t = threadIdx.x % PB, g = threadIdx.x / PB;
    for (int h = 0; h < nh; h++) {
      u64 m = 0;
      unsigned c = 0;
#pragma unroll
      for (int r = g * (kCl / G); r < (g + 1) * (kCl / G); r++) {
        m += cl.map_shared_rank(s.hm, r)[h * kBins + rank * PB + t];
        c += cl.map_shared_rank(s.hc, r)[h * kBins + rank * PB + t];
      }
      x.rs_m[h][threadIdx.x] = m;
      x.rs_c[h][threadIdx.x] = c;
    }
  }
  __syncthreads();
  for (int h = 0; h < nh; h++) {
    u64 m = 0;
    unsigned c = 0;
    if (threadIdx.x < PB) {
#pragma unroll
      for (int g = 0; g < G; g++) {
        m += x.rs_m[h][g * PB + threadIdx.x];
        c += x.rs_c[h][g * PB + threadIdx.x];
      }
      x.pm[h][threadIdx.x] = m;
      x.pc[h][threadIdx.x] = c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      m += __shfl_xor_sync(0xffffffffu, m, o);
      c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    if (lane == 0) {
      s_wt[warp] = m;
      s_wc[warp] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      u64 tm = 0;
      unsigned tc = 0;
      for (int w = 0; w < (PB + 31) / 32; w++) {
        tm += s_wt[w];
        tc += s_wc[w];
      }
      x.port_m[h] = tm;
      x.port_c[h] = tc;
    }
    __syncthreads();
  }
  cl.sync();
  // the portion each target falls in (portions in descending order): warp i
  // for target i, lane L reads portion kCl-1-L
  if (warp < 2) {
    const int i = warp, h = two ? i : 0;
    u64 pm = 0;
    unsigned pc = 0;
    if (lane < kCl) {
      pm = *cl.map_shared_rank(&x.port_m[h], kCl - 1 - lane);
      pc = *cl.map_shared_rank(&x.port_c[h], kCl - 1 - lane);
    }
    u64 incl = pm;
#pragma unroll
    for (int o = 1; o < kCl; o <<= 1) {
      const u64 u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    const u64 above = cut[i].above;
    const unsigned cr = __ballot_sync(0xffffffffu, lane < kCl && above + incl > target[i]);
    const unsigned ne = __ballot_sync(0xffffffffu, lane < kCl && pc > 0);
    const u64 total = __shfl_sync(0xffffffffu, incl, kCl - 1);
    const int L = cr ? __ffs(cr) - 1 : 0;
    const u64 before = __shfl_sync(0xffffffffu, incl - pm, L);
    const u64 pm_low = __shfl_sync(0xffffffffu, pm, ne ? 31 - __clz(ne) : 0);
    if (lane == 0) {
      if (cr) {
        s_q[i] = kCl - 1 - L;
        s_cr[i] = 1;
        s_acc[i] = above + before;  // mass above the portion
      } else {
        // none crossed: the lowest non-empty portion
        s_q[i] = ne ? kCl - 1 - (31 - __clz(ne)) : -1;
        s_cr[i] = 0;
        s_acc[i] = above + total - pm_low;
      }
    }
  }
  __syncthreads();
  {
    // half i = threadIdx.x / 256 walks target i; its thread tt < PB holds
    // bin q*PB + PB-1-tt (descending)
    const int i = threadIdx.x >> 8, tt = threadIdx.x & 255, h = two ? i : 0;
    const int q = s_q[i];
    const bool crossed = s_cr[i] != 0;
    const u64 base = s_acc[i];
    u64 m = 0;
    unsigned c = 0;
    if (q >= 0 && tt < PB) {
      m = cl.map_shared_rank(&x.pm[h][0], q)[PB - 1 - tt];
      c = cl.map_shared_rank(&x.pc[h][0], q)[PB - 1 - tt];
    }
    u64 incl = m;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const u64 u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) s_wt[warp] = incl;
    __syncthreads();
    for (int w = i * 8; w < warp; w++) incl += s_wt[w];
    const unsigned cr = __ballot_sync(0xffffffffu, tt < PB && base + incl > target[i]);
    const unsigned ne = __ballot_sync(0xffffffffu, tt < PB && c > 0);
    if (lane == 0) {
      s_first[warp] = cr ? (warp & 7) * 32 + __ffs(cr) - 1 : INT_MAX;
      s_last[warp] = ne ? (warp & 7) * 32 + 31 - __clz(ne) : -1;
    }
    __syncthreads();
    int first = INT_MAX, last = -1;
    for (int w = i * 8; w < i * 8 + 8; w++) {
      first = min(first, s_first[w]);
      last = max(last, s_last[w]);
    }
    const int pick = crossed ? first : last;
    if (q < 0) {
      if (tt == 0) s_cut[i] = Cut{cut[i].prefix, cut[i].above, 0u};
    } else if (tt == pick) {
      s_cut[i] = Cut{cut[i].prefix | ((unsigned)(q * PB + PB - 1 - tt) << shift),
                     base + incl - m, c};
    }
  }
  __syncthreads();
  cut[0] = s_cut[0];
  cut[1] = s_cut[1];
  __syncthreads();
}

// Radix selection over the cluster for two targets: the probability at which
// the mass in descending order first exceeds each target (the smallest
// probability if none does).  Probabilities are positive, so bit 31 is
// zero: passes over bits 30-20, 19-9 and 8-0.  FIRST: see radix_pass.
template <bool FIRST>
__device__ void cluster_mass_select(const Slice& s, Exchange& x, cg::cluster_group& cl,
                                    const u64* target, Cut* cut, float sum) {
  cut[0] = Cut{0u, 0ull, 0u};
  cut[1] = Cut{0u, 0ull, 0u};
  radix_pass<2048, FIRST>(s, x, cl, 20, 0u, target, cut, sum);
  SAMPLE_MARK(10);
  radix_pass<2048, false>(s, x, cl, 9, 0x7ff00000u, target, cut, sum);
  SAMPLE_MARK(11);
  radix_pass<512, false>(s, x, cl, 0, 0x7ffffe00u, target, cut, sum);
}

// Which histogram of the last pass holds target i's final bin.
__device__ __forceinline__ int last_hist(const Cut* cut, int i) {
  return i == 1 && (cut[0].prefix & 0x7ffffe00u) != (cut[1].prefix & 0x7ffffe00u) ? 1 : 0;
}

// Within this CTA's slice: the index (global) of the k-th element, in index
// order, whose probability has bit pattern `key`.  Warp w scans its
// contiguous range.
__device__ int slice_kth(const Slice& s, unsigned key, long long k) {
  __shared__ unsigned s_w[kWarps];
  __shared__ int s_idx;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int pw = ((s.len + kWarps - 1) / kWarps + 31) & ~31;
  const int w0 = warp * pw, w1 = min(s.len, w0 + pw);
  unsigned c = 0;
  for (int i = w0 + lane; i < w1; i += 32) c += __float_as_uint(s.p[i]) == key ? 1u : 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if (lane == 0) s_w[warp] = c;
  if (threadIdx.x == 0) s_idx = -1;
  __syncthreads();
  long long base = 0;
  int tw = -1;
  for (int w = 0; w < kWarps; w++) {
    if (k < base + s_w[w]) {
      tw = w;
      break;
    }
    base += s_w[w];
  }
  if (warp == tw) {
    for (int i0 = w0; i0 < w1; i0 += 32) {
      const int i = i0 + lane;
      const unsigned bal = __ballot_sync(0xffffffffu, i < w1 && __float_as_uint(s.p[i]) == key);
      const int pc = __popc(bal);
      if (k < base + pc) {
        if (lane == 0) s_idx = s.c0 + i0 + (int)__fns(bal, 0, (int)(k - base) + 1);
        break;
      }
      base += pc;
    }
  }
  __syncthreads();
  return s_idx;
}

// Over the cluster: the k-th element, in index order, with probability bits
// `key`; each CTA's count of them is bin `key & 511` of its histogram h
// from the last pass.  The CTA that holds it writes *out.
__device__ void cluster_kth(const Slice& s, cg::cluster_group& cl, unsigned key, int h,
                            long long k, int* out) {
  long long base = 0, mine = 0;
  int owner = -1;
  for (int r = 0; r < kCl; r++) {
    const unsigned rc = cl.map_shared_rank(s.hc, r)[h * kBins + (int)(key & 511u)];
    if (owner < 0 && k < base + rc) {
      owner = r;
      mine = base;
    }
    if (owner < 0) base += rc;
  }
  if (owner == (int)cl.block_rank()) {
    const int idx = slice_kth(s, key, k - mine);
    if (threadIdx.x == 0 && idx >= 0) *out = idx;
  }
}

__device__ Slice slice_of(const SampleArgs& a, float* smem, int rank) {
  Slice s;
  const int per = (a.n + kCl - 1) / kCl;
  s.c0 = rank * per;
  s.len = max(0, min(per, a.n - s.c0));
  s.hm = reinterpret_cast<u64*>(smem);
  s.hc = reinterpret_cast<unsigned*>(s.hm + 2 * kBins);
  s.p = reinterpret_cast<float*>(s.hc + 2 * kBins);
  return s;
}

__device__ void load_row(const Slice& s, const float* row) {
  for (int i = threadIdx.x; i < s.len; i += kThr) s.p[i] = row[s.c0 + i];
}

// The cluster's max m of the slice, then p <- expf((p - m) / t); returns the
// cluster's sum of those (per-CTA double sums added in rank order, then
// rounded to float).
__device__ float cluster_exp(const Slice& s, Exchange& x, cg::cluster_group& cl, float t) {
  __shared__ float s_f[kWarps];
  __shared__ double s_d[kWarps];
  __shared__ float s_m, s_sum;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float m = -INFINITY;
  for_slice(s, [&](int, float v) { m = fmaxf(m, v); });
  m = block_reduce(m, s_f, [](float a, float b) { return fmaxf(a, b); });
  if (threadIdx.x == 0) x.mx = m;
  cl.sync();
  if (warp == 0) {
    float v = lane < kCl ? *cl.map_shared_rank(&x.mx, lane) : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) s_m = v;
  }
  __syncthreads();
  m = s_m;
  double sd = 0.0;
  float* pw = s.p;
  for_slice(s, [&](int i, float v) {
    const float e = expf(__fdiv_rn(__fsub_rn(v, m), t));
    pw[i] = e;
    sd += (double)e;
  });
  sd = block_reduce(sd, s_d, [](double a, double b) { return a + b; });
  if (threadIdx.x == 0) x.sum = sd;
  cl.sync();
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int r = 0; r < kCl; r++) tot += *cl.map_shared_rank(&x.sum, r);
    s_sum = (float)tot;
  }
  __syncthreads();
  return s_sum;
}

__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kThr, 1)
    sample_top_p_kernel(SampleArgs a) {
  extern __shared__ __align__(16) float smem[];
  __shared__ Exchange x;
  cg::cluster_group cl = cg::this_cluster();
  const int row = blockIdx.x / kCl, rank = (int)cl.block_rank();
  float* l = a.logits + (long)row * a.n;
  SAMPLE_MARK(0);
  const Slice s = slice_of(a, smem, rank);
  load_row(s, l);
  __syncthreads();
  // 1. repetition penalty (every occurrence), 2. UNK blocked; the penalised
  // logits are written back, as the reference modifies its buffer
  if (a.history) {
    const int* hist = a.history + (long)row * a.history_stride;
    const int hn = a.history_len[row];
    for (int j = threadIdx.x; j < hn; j += kThr) {
      const int t = hist[j] - s.c0;
      if (t >= 0 && t < s.len) penalise_shared(s.p + t, a.penalty);
    }
  }
  __syncthreads();
  if (a.block0 && rank == 0 && threadIdx.x == 0 && s.len > 0) s.p[0] = -1e9f;
  __syncthreads();
  if (a.history || a.block0)
    for (int i = threadIdx.x; i < s.len; i += kThr) l[s.c0 + i] = s.p[i];
  SAMPLE_MARK(1);
  // 3. softmax (the division by the sum happens in the first radix pass)
  const float sum = cluster_exp(s, x, cl, a.temperature);
  SAMPLE_MARK(2);
  // 4. and 5.: the nucleus' cut (target top) and the draw's (target
  // r * top, checked below against the exact r * cum)
  const float rr = a.r[row];
  const u64 top = (u64)((double)a.top_p * kFix);
  u64 target[2] = {top, (u64)((double)rr * (double)top)};
  Cut cut[2];
  cluster_mass_select<true>(s, x, cl, target, cut, sum);
  SAMPLE_MARK(3);
  const unsigned tau = cut[0].prefix;
  const u64 ftau = fix(__uint_as_float(tau)) ? fix(__uint_as_float(tau)) : 1ull;
  long long j = top >= cut[0].above ? (long long)((top - cut[0].above) / ftau) + 1 : 1;
  if (j > (long long)cut[0].cnt) j = cut[0].cnt;
  if (j < 1) j = 1;
  const u64 cum = cut[0].above + (u64)j * ftau;
  const u64 draw = (u64)((double)rr * (double)cum);
  int* out = a.out + row;
  if (draw >= cut[0].above) {
    // among the tied elements at the nucleus' cut
    long long k = (long long)((draw - cut[0].above) / ftau);
    if (k >= j) k = j - 1;
    cluster_kth(s, cl, tau, 0, k, out);
  } else {
    // above the cut: the first element of the whole descending order whose
    // running sum exceeds the draw
    Cut d = cut[1];
    int h = last_hist(cut, 1);
    u64 fv = fix(__uint_as_float(d.prefix)) ? fix(__uint_as_float(d.prefix)) : 1ull;
    if (!(d.above <= draw && draw - d.above < (u64)d.cnt * fv)) {
      SAMPLE_MARK(4);
      const u64 t2[2] = {draw, draw};
      Cut c2[2];
      cluster_mass_select<false>(s, x, cl, t2, c2, sum);
      d = c2[0];
      h = 0;
      fv = fix(__uint_as_float(d.prefix)) ? fix(__uint_as_float(d.prefix)) : 1ull;
    }
    long long k = draw >= d.above ? (long long)((draw - d.above) / fv) : 0;
    if (k >= (long long)d.cnt) k = (long long)d.cnt - 1;
    if (k < 0) k = 0;
    cluster_kth(s, cl, d.prefix, h, k, out);
  }
  SAMPLE_MARK(5);
  cl.sync();  // keep this CTA's shared memory alive for the others' reads
  SAMPLE_MARK(6);
}

// sample_temperature (sampler_temp.c:96-115): softmax at the temperature,
// then the first index, in index order, whose running sum exceeds the draw
// r (sample_from_probs, sampler_temp.c:74-94), with running sums in 2^-50
// fixed point.  A draw above the whole mass (the reference then returns n,
// one past the vocabulary) gives n - 1.
__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kThr, 1)
    sample_temperature_kernel(SampleArgs a) {
  extern __shared__ __align__(16) float smem[];
  __shared__ Exchange x;
  __shared__ u64 s_w[kWarps];
  __shared__ u64 s_red[kWarps];
  __shared__ int s_idx;
  cg::cluster_group cl = cg::this_cluster();
  const int row = blockIdx.x / kCl, rank = (int)cl.block_rank();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const Slice s = slice_of(a, smem, rank);
  load_row(s, a.logits + (long)row * a.n);
  __syncthreads();
  const float sum = cluster_exp(s, x, cl, a.temperature);
  float* pw = s.p;
  u64 m = 0;
  for_slice(s, [&](int i, float e) {
    const float p = __fdiv_rn(e, sum);
    pw[i] = p;
    m += fix(p);
  });
  const u64 target = (u64)((double)a.r[row] * kFix);
  m = block_reduce(m, s_red, [](u64 p, u64 q) { return p + q; });
  if (threadIdx.x == 0) x.tm = m;
  cl.sync();
  u64 base = 0;
  int owner = -1;
  for (int r = 0; r < kCl; r++) {
    const u64 rm = *cl.map_shared_rank(&x.tm, r);
    if (base + rm > target) {
      owner = r;
      break;
    }
    base += rm;
  }
  if (owner < 0) {
    if (rank == kCl - 1 && threadIdx.x == 0) a.out[row] = a.n - 1;
  } else if (owner == rank) {
    const int pwid = ((s.len + kWarps - 1) / kWarps + 31) & ~31;
    const int w0 = warp * pwid, w1 = min(s.len, w0 + pwid);
    u64 wm = 0;
    for (int i = w0 + lane; i < w1; i += 32) wm += fix(s.p[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wm += __shfl_xor_sync(0xffffffffu, wm, o);
    if (lane == 0) s_w[warp] = wm;
    if (threadIdx.x == 0) s_idx = -1;
    __syncthreads();
    int tw = -1;
    for (int w = 0; w < kWarps; w++) {
      if (base + s_w[w] > target) {
        tw = w;
        break;
      }
      base += s_w[w];
    }
    if (warp == tw) {
      for (int i0 = w0; i0 < w1; i0 += 32) {
        const int i = i0 + lane;
        u64 v = i < w1 ? fix(s.p[i]) : 0ull;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const u64 u = __shfl_up_sync(0xffffffffu, v, o);
          if (lane >= o) v += u;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, i < w1 && base + v > target);
        if (hit) {
          if (lane == 0) s_idx = s.c0 + i0 + __ffs(hit) - 1;
          break;
        }
        base += __shfl_sync(0xffffffffu, v, 31);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) a.out[row] = s_idx >= 0 ? s_idx : a.n - 1;
  }
  cl.sync();
}

int launch_sample(bool top_p, const SampleArgs& a, int rows, cudaStream_t st) {
  const int per = (a.n + kCl - 1) / kCl;
  if (per > kMaxSlice) {
    ec_set_last_error("vocabulary too large for device sampling");
    return EC_ERR_UNSUPPORTED;
  }
  const size_t smem = kHistBytes + (size_t)((per + 3) & ~3) * 4;
  const void* k = top_p ? (const void*)sample_top_p_kernel : (const void*)sample_temperature_kernel;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) {
    if (top_p)
      sample_top_p_kernel<<<rows * kCl, kThr, smem, st>>>(a);
    else
      sample_temperature_kernel<<<rows * kCl, kThr, smem, st>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    ec_set_last_error(cudaGetErrorString(e));
    return EC_ERR_CUDA;
  }
  return EC_OK;
}

}  // namespace
}  // namespace ec

extern "C" int ec_op_sample_top_p(float* logits, int n, int rows, const int* history,
                                  const int* history_len, int history_stride, float temperature,
                                  float top_p, float penalty, int block_token0, const float* r,
                                  int* out, void* stream) {
  if (!logits || !r || !out || n <= 0 || rows <= 0 || !(temperature > 0.0f) ||
      !(top_p > 0.0f) || !(penalty > 0.0f) || (history && !history_len)) {
    ec_set_last_error("bad argument");
    return EC_ERR_ARG;
  }
  ec::SampleArgs a{logits, n, history, history_len, history_stride, temperature, top_p, penalty,
                   block_token0, r, out};
  return ec::launch_sample(true, a, rows, static_cast<cudaStream_t>(stream));
}

extern "C" int ec_op_sample_temperature(const float* logits, int n, int rows, float temperature,
                                        const float* r, int* out, void* stream) {
  if (!logits || !r || !out || n <= 0 || rows <= 0 || !(temperature > 0.0f)) {
    ec_set_last_error("bad argument");
    return EC_ERR_ARG;
  }
  ec::SampleArgs a{const_cast<float*>(logits), n, nullptr, nullptr, 0, temperature, 1.0f, 1.0f,
                   0, r, out};
  return ec::launch_sample(false, a, rows, static_cast<cudaStream_t>(stream));
}

#ifdef EC_PHASE_TIMING
extern "C" int ec_debug_sample_times(long long* out) {
  return cudaMemcpyFromSymbol(out, ec::g_sample_ts, sizeof(ec::g_sample_ts)) == cudaSuccess ? 0
                                                                                             : -2;
}
#endif
