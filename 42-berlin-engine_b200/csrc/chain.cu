// chain.cu -- the decode step's weight-streaming GEMVs of one layer as ONE
// persistent kernel: the attention output projection (+ residual), the
// gate/up projection (RMSNorm prologue, SwiGLU epilogue), the down projection
// (+ residual) and the next layer's QKV projection (RMSNorm prologue) -- or,
// after the last layer, the LM head.
//
// Arithmetic, weight layout and the per-thread mapping are those of
// gemv_packed.cu (the reference's matvec_bf16_f32_blocked order, bit for
// bit).  What changes is the schedule: one CTA per SM owns a fixed range of
// rows of every matrix; its producer warp streams all of those rows, phase
// after phase, through one ring of stages without ever waiting for
// activations (weights do not depend on them), while the consumer warps wait
// for each phase's input vector -- complete only when every CTA has finished
// the previous phase -- through a grid-wide counter.  The weight stream
// therefore never stops at a matrix boundary: it keeps HBM busy through the
// epilogue, the wait and the RMSNorm that separate two matrices.
//
// All CTAs must be resident at once (one per SM, grid = SM count).  Waits are
// bounded: a wait that runs out sets the error word and the CTA stops
// computing.  The phase counters return to zero when the last CTA leaves.
#include "chain.cuh"
#include "ec_internal.cuh"

namespace ec {

#ifdef EC_PHASE_TIMING
__device__ long long g_chain_ts[64];
#define CHAIN_MARK(cond, s)                                                 \
  do {                                                                      \
    if (cond) {                                                             \
      long long t_;                                                         \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));               \
      g_chain_ts[s] = t_;                                                   \
    }                                                                       \
  } while (0)
#else
#define CHAIN_MARK(cond, s) \
  do {                      \
  } while (0)
#endif

namespace {

// -(2^23 + 128), twice: the INT8 decode bias
constexpr uint64_t kBias2 = 0xCB000080CB000080ull;
constexpr int kStagesMax = 8;
constexpr int kWarps = 16;  // consumer warps; one row quad each per stage

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// This CTA's share of one phase: row quads [q0, q1) in ngroups groups of qs
// quads (the same qs on every CTA: the fewest groups of at most kWarps quads,
// evenly filled, so no CTA ends on a near-empty group), and m chunks per ring
// slot (narrow groups carry several chunks so a slot still moves ~32 KB).
struct Split {
  int nq, q0, q1, qs, ngroups, nchunks, m;
};
template <int KCE>
__device__ __forceinline__ Split split_t(const ChainPhase& ph, int b, int G) {
  Split r;
  r.nq = (ph.N + 3) >> 2;
  r.q0 = (int)((long)r.nq * b / G);
  r.q1 = (int)((long)r.nq * (b + 1) / G);
  const int qmax = (r.nq + G - 1) / G;
  const int gmax = (qmax + kWarps - 1) / kWarps;
  r.qs = (qmax + gmax - 1) / gmax;
  r.ngroups = (r.q1 - r.q0 + r.qs - 1) / r.qs;
  r.nchunks = ph.K / KCE;
  r.m = kWarps / r.qs;
  if (r.m < 1) r.m = 1;
  if (r.m > r.nchunks) r.m = r.nchunks;
  return r;
}

// RMSNorm of xs[0..K) in place with the norm weights already in shared
// memory: rmsnorm_f32_avx2 (ops_norm.c:105-124) -- lane l of 8 sums x[j]^2
// over j = l (mod 8) with one fused multiply-add per element, in order; the
// lanes' sums are added by hsum8, the scalar tail follows.  The 8 summing
// threads load their elements 32 at a time ahead of the chain, so the
// sum costs the chain of dependent FMAs rather than a shared-memory latency
// per element (padding with zeros adds +0 to a non-negative sum: exact).
__device__ __forceinline__ void rmsnorm_chain(float* xs, const uint16_t* wn, int K, float eps,
                                              float* red, int ct, int nc) {
  if (ct < 8) {
    constexpr int B = 32;
    const int n8 = K >> 3;
    const float* xl = xs + ct;
    float acc = 0.0f, cur[B], nxt[B];
#pragma unroll
    for (int b = 0; b < B; b++) cur[b] = b < n8 ? xl[8 * b] : 0.0f;
    for (int base = 0; base < n8; base += B) {
#pragma unroll
      for (int b = 0; b < B; b++) nxt[b] = base + B + b < n8 ? xl[8 * (base + B + b)] : 0.0f;
#pragma unroll
      for (int b = 0; b < B; b++) acc = __fmaf_rn(cur[b], cur[b], acc);
#pragma unroll
      for (int b = 0; b < B; b++) cur[b] = nxt[b];
    }
    red[ct] = acc;
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nc));
  if (ct == 0) {
    float ss = hsum8(red);
    for (int j = K & ~7; j < K; j++) ss = __fmaf_rn(xs[j], xs[j], ss);
    ss = __fdiv_rn(ss, (float)K);
    red[8] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, eps)));
  }
  asm volatile("bar.sync 1, %0;" ::"r"(nc));
  const float inv = red[8];
  for (int j = ct; j < K; j += nc) xs[j] = __fmul_rn(__fmul_rn(xs[j], inv), bf16_to_f32(wn[j]));
  asm volatile("bar.sync 1, %0;" ::"r"(nc));
}

template <int WK, int KCE>
__global__ void __launch_bounds__(32 + 32 * kWarps, 1) gemv_chain_kernel(ChainParams P) {
  auto split = [](const ChainPhase& ph, int b, int G) { return split_t<KCE>(ph, b, G); };
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = P.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStagesMax;
  uint64_t* xbar = empty + kStagesMax;
  float* red = reinterpret_cast<float*>(xbar + 2);  // 16 floats
  float* xs = red + 16;                              // [kmax]
  uint16_t* wn = reinterpret_cast<uint16_t*>(xs + P.kmax);  // [knorm] norm weights
  uint8_t* stages = reinterpret_cast<uint8_t*>(wn) + ((P.knorm * 2 + 15) & ~15);
  constexpr int QS = kWarps;  // quads per stage
  constexpr int stage_bytes = QS * 4 * KCE;
  __shared__ int s_go;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  const bool mk = P.mark && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1);
  const int mb = blockIdx.x == 0 ? 0 : 32;
  (void)mk;
  (void)mb;
  CHAIN_MARK(mk && tid == 0, mb);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int t = 0;
      for (int p = 0; p < P.nph; p++) {
        const ChainPhase& ph = P.ph[p];
        const Split sp = split(ph, blockIdx.x, G);
        for (int g = 0; g < sp.ngroups; g++) {
          const int gq0 = sp.q0 + g * sp.qs, gn = min(sp.qs, sp.q1 - gq0);
          for (int c0 = 0; c0 < sp.nchunks; c0 += sp.m, t++) {
            const int s = t % S, mc = min(sp.m, sp.nchunks - c0);
            if (t >= S && !mbar_wait(&empty[s], ((t / S) - 1) & 1, P.err)) return;
            const uint32_t bytes = (uint32_t)gn * 4 * KCE;
            mbar_expect_tx(&full[s], bytes * mc);
            for (int i = 0; i < mc; i++)
              bulk_g2s(stages + (size_t)s * stage_bytes + (size_t)i * bytes,
                       ph.w + ((long)(c0 + i) * sp.nq + gq0) * 4 * KCE, bytes, &full[s]);
          }
        }
      }
      CHAIN_MARK(mk, mb + 20);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int ct = tid - 32, wc = warp - 1, nc = kWarps * 32;
  const int rq = lane >> 3, sl = lane & 7;
  bool ok = true, live = true;
  int t = 0;
  for (int p = 0; p < P.nph; p++) {
    const ChainPhase& ph = P.ph[p];
    // ---- the input vector: complete once every CTA finished phase p-1
    if (p == 0) {
      pdl_wait();
    } else {
      if (ct == 0) {
        bool got = false;
        const uint32_t lim = P.wait_iters > 0 ? (uint32_t)P.wait_iters : kWaitLimit;
        const int need = G + (p == 1 ? P.wait_extra : 0);
        for (uint32_t it = 0; it < lim && ok; it++)
          if (ld_acquire(P.ctr + p - 1) >= need) {
            got = true;
            break;
          } else {
            __nanosleep(64);
          }
        if (!got && ok) atomicCAS(P.err, 0, EC_ERR_TIMEOUT);
        s_go = got && ok;
        fence_proxy_async();
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nc));
      ok = ok && s_go;
    }
    CHAIN_MARK(mk && ct == 0, mb + 1 + 2 * p);
    if (ct == 0 && ok) {
      // the vector and, for an RMSNorm prologue, its weights
      const bool nw = ph.pro == PRO_RMSNORM;
      mbar_expect_tx(xbar, (uint32_t)(ph.K * 4 + (nw ? ph.K * 2 : 0)));
      bulk_g2s(xs, ph.x, (uint32_t)(ph.K * 4), xbar);
      if (nw) bulk_g2s(wn, ph.norm_w, (uint32_t)(ph.K * 2), xbar);
    }
    if (ok) ok = mbar_wait(xbar, p & 1, P.err);
    CHAIN_MARK(mk && ct == 0 && p < 4, mb + 10 + p);
    if (ph.pro == PRO_RMSNORM && ok) rmsnorm_chain(xs, wn, ph.K, P.eps, red, ct, nc);
    CHAIN_MARK(mk && ct == 0 && p < 4, mb + 14 + p);

    // ---- this CTA's rows, group by group, slot by slot
    const Split sp = split(ph, blockIdx.x, G);
    for (int g = 0; g < sp.ngroups; g++) {
      const int gq0 = sp.q0 + g * sp.qs, gn = min(sp.qs, sp.q1 - gq0);
      uint64_t acc01 = 0, acc23 = 0;
      for (int c0 = 0; c0 < sp.nchunks; c0 += sp.m, t++) {
        const int s = t % S, mc = min(sp.m, sp.nchunks - c0);
        // every slot is waited for, also after a failed wait: no bulk copy
        // may still be landing in shared memory when the CTA exits.  A slot
        // that never fills after a failure means the producer stopped: no
        // later slot has a copy either.
        bool landed = false;
        if (live) landed = mbar_wait(&full[s], (t / S) & 1, ok ? P.err : nullptr);
        if (!landed) {
          if (!ok) live = false;
          ok = false;
        }
        if (ok && wc < gn) {
          for (int i = 0; i < mc; i++) {
            const uint8_t* base = stages + (size_t)s * stage_bytes + (size_t)(i * gn + wc) * 4 * KCE +
                                  rq * 32 + sl * 4;
            const float* xc = xs + (c0 + i) * KCE + sl * 4;
#pragma unroll
            for (int pc = 0; pc < KCE / 32; pc++) {
              const ulonglong2 xv = *reinterpret_cast<const ulonglong2*>(xc + pc * 32);
              const uint32_t wv = *reinterpret_cast<const uint32_t*>(base + pc * 128);
              if constexpr (WK == EC_W_INT8) {
                fma4_i8(wv, xv.x, xv.y, kBias2, acc01, acc23);
              } else {
                uint64_t w01, w23;
                decode_pairs<WK>(wv, w01, w23);
                fma2(acc01, w01, xv.x);
                fma2(acc23, w23, xv.y);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // combine lanes: (g0+g1)+(g2+g3) per 8-lane position, then hsum8
      float v[4] = {lo_f(acc01), hi_f(acc01), lo_f(acc23), hi_f(acc23)};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float t1 = __fadd_rn(v[k], __shfl_xor_sync(0xffffffffu, v[k], 2));
        v[k] = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 4));
      }
#pragma unroll
      for (int k = 0; k < 4; k++) v[k] = __fadd_rn(v[k], __shfl_xor_sync(0xffffffffu, v[k], 1));
      float sum = __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
      const int gr = (gq0 + wc) * 4 + rq;
      const bool valid = ok && wc < gn && gr < ph.N;
      if (valid) sum = __fmul_rn(sum, ph.scale[gr]);
      if (ph.epi == EPI_SWIGLU) {
        const float up = __shfl_down_sync(0xffffffffu, sum, 8);
        if (valid && sl == 0 && (rq & 1) == 0) {
          const int o = gr >> 1;
          float sig;
          if (o < ph.silu_vec_limit)
            sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf_vec(__fsub_rn(0.0f, sum))));
          else
            sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf(-sum)));
          ph.y[o] = __fmul_rn(__fmul_rn(sum, sig), up);
        }
      } else if (ph.epi == EPI_RESID) {
        if (valid && sl == 0) ph.y[gr] = __fadd_rn(ph.y[gr], sum);
      } else {
        if (valid && sl == 0) ph.y[gr] = sum;
      }
    }
    // ---- phase done on this CTA: publish (release) for every other CTA
    asm volatile("bar.sync 1, %0;" ::"r"(nc));
    CHAIN_MARK(mk && ct == 0, mb + 2 + 2 * p);
    if (ct == 0) {
      fence_proxy_async();
      __threadfence();
      atomicAdd(P.ctr + p, 1);
    }
  }
  // the last CTA out returns the counters to zero for the next step
  if (ct == 0) {
    __threadfence();
    if (atomicAdd(P.ctr + kMaxChainPhases, 1) == G - 1) {
      for (int p = 0; p <= kMaxChainPhases; p++) atomicExch(P.ctr + p, 0);
    }
  }
}

// ---------------------------------------------------------------------------
// Batched chain: NB sequences (2..8) share one pass over the weights.  Each
// ring slot carries one 512-column chunk of a group of row quads AND the same
// chunk of every sequence's input vector; a weight word is decoded once and
// accumulated into NB sets of lane accumulators, each in the reference's
// order, so every sequence's result is bit-identical to its batch-1 result.
// The producer issues weight copies as far ahead as the ring allows, across
// phase boundaries; a slot's vector copies go out only once that phase's
// input is complete (grid counter), so the weight stream never waits for
// activations.  RMSNorm runs as its own phase (PRO_NORM_ROWS): CTA b stages
// row b, runs the reference's 8-lane sum of squares and writes the
// normalised row, which the next phase streams.
template <int WK, int NB>
__global__ void __launch_bounds__(32 + 32 * kWarps, 1) gemv_chain_nb_kernel(ChainParams P) {
  constexpr int KCE = 512;
  constexpr int kWB = kWarps * 4 * KCE;  // weight bytes per slot
  constexpr int kXB = NB * KCE * 4;      // vector bytes per slot
  constexpr int kSlot = kWB + kXB;
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = P.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStagesMax;
  uint64_t* rbar = empty + kStagesMax;
  float* red = reinterpret_cast<float*>(rbar + 2);  // 16 floats
  float* rowbuf = reinterpret_cast<float*>(smem + 512);     // [kmax] (norm rows)
  uint8_t* ring = smem + 512 + ((P.kmax * 4 + 127) & ~127);
  __shared__ int s_go;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_init(rbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    struct Cur {
      int p = 0, g = 0, c = 0;
      int sp_p = -1;  // phase whose split is cached
      Split sp;
    };
    // first task at or after u (skipping phases without weights); false at end
    auto settle = [&](Cur& u) -> bool {
      while (u.p < P.nph) {
        const ChainPhase& ph = P.ph[u.p];
        if (ph.pro != PRO_NORM_ROWS) {
          if (u.sp_p != u.p) {
            u.sp = split_t<KCE>(ph, blockIdx.x, G);
            u.sp_p = u.p;
          }
          if (u.g < u.sp.ngroups) return true;
        }
        u.p++;
        u.g = u.c = 0;
      }
      return false;
    };
    auto advance = [&](Cur& u) {
      if (++u.c == u.sp.nchunks) {
        u.c = 0;
        u.g++;
      }
    };
    Cur cw, cx;  // next weight copy, next vector copy
    int t = 0, tx = 0, ready = -1;
    bool have_w = settle(cw), have_x = settle(cx);
    uint32_t idle = 0;
    while (have_x) {
      // weights for task t when its slot is free
      if (have_w) {
        const int s = t % S;
        if (t < S || mbar_test(&empty[s], ((t / S) - 1) & 1)) {
          const ChainPhase& ph = P.ph[cw.p];
          const Split& sp = cw.sp;
          const int gq0 = sp.q0 + cw.g * sp.qs, gn = min(sp.qs, sp.q1 - gq0);
          const uint32_t wb = (uint32_t)gn * 4 * KCE;
          mbar_expect_tx(&full[s], wb + kXB);
          bulk_g2s(ring + (size_t)s * kSlot, ph.w + ((long)cw.c * sp.nq + gq0) * 4 * KCE, wb,
                   &full[s]);
          t++;
          advance(cw);
          have_w = settle(cw);
          idle = 0;
          continue;
        }
      }
      // vectors for task tx once its phase's input is complete
      if (tx < t) {
        if (cx.p > ready) {
          if (cx.p == 0) {
            pdl_wait();  // the previous kernel wrote phase 0's input
          } else if (ld_acquire(P.ctr + cx.p - 1) < G) {
            if (++idle > (kWaitLimit << 4)) {
              atomicCAS(P.err, 0, EC_ERR_TIMEOUT);
              return;
            }
            __nanosleep(64);
            continue;
          }
          fence_proxy_async();
          ready = cx.p;
        }
        const ChainPhase& ph = P.ph[cx.p];
        const int s = tx % S;
        uint8_t* xd = ring + (size_t)s * kSlot + kWB;
#pragma unroll
        for (int b = 0; b < NB; b++)
          bulk_g2s(xd + b * KCE * 4, ph.x + (long)b * ph.x_stride + (long)cx.c * KCE, KCE * 4,
                   &full[s]);
        tx++;
        advance(cx);
        have_x = settle(cx);
        idle = 0;
        continue;
      }
      if (++idle > (kWaitLimit << 4)) {
        atomicCAS(P.err, 0, EC_ERR_TIMEOUT);
        return;
      }
      __nanosleep(64);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int ct = tid - 32, wc = warp - 1, nc = kWarps * 32;
  const int rq = lane >> 3, sl = lane & 7;
  bool ok = true;
  int t = 0, nrm = 0;  // nrm: norm phases so far (rbar's phase parity)
  for (int p = 0; p < P.nph; p++) {
    const ChainPhase& ph = P.ph[p];
    if (ph.pro == PRO_NORM_ROWS) {
      // wait for the input, then CTA b normalises row b
      if (p == 0) pdl_wait();
      if (ct == 0) {
        bool got = p == 0;
        for (uint32_t it = 0; it < kWaitLimit && ok && !got; it++) {
          if (ld_acquire(P.ctr + p - 1) >= G) got = true;
          else __nanosleep(64);
        }
        if (!got && ok) atomicCAS(P.err, 0, EC_ERR_TIMEOUT);
        s_go = got && ok;
        fence_proxy_async();
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nc));
      ok = ok && s_go;
      const int b = blockIdx.x;
      if (b < NB && ok) {
        if (ct == 0) {
          mbar_expect_tx(rbar, (uint32_t)(ph.K * 4));
          bulk_g2s(rowbuf, ph.x + (long)b * ph.x_stride, (uint32_t)(ph.K * 4), rbar);
        }
        ok = mbar_wait(rbar, nrm & 1, P.err);
        if (ok) rmsnorm_smem(rowbuf, ph.norm_w, ph.K, P.eps, red, ct, nc);
        float* y = ph.y + (long)b * ph.y_stride;
        for (int j = ct; j < ph.K && ok; j += nc) y[j] = rowbuf[j];
      }
      nrm++;
    } else {
      if (p == 0) pdl_wait();  // the epilogue may read what earlier kernels wrote
      const Split sp = split_t<KCE>(ph, blockIdx.x, G);
      for (int g = 0; g < sp.ngroups; g++) {
        const int gq0 = sp.q0 + g * sp.qs, gn = min(sp.qs, sp.q1 - gq0);
        uint64_t acc01[NB], acc23[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) acc01[b] = acc23[b] = 0;
        for (int c = 0; c < sp.nchunks; c++, t++) {
          const int s = t % S;
          if (ok) ok = mbar_wait(&full[s], (t / S) & 1, P.err);
          if (ok && wc < gn) {
            const uint8_t* wbase = ring + (size_t)s * kSlot + (size_t)wc * 4 * KCE + rq * 32 + sl * 4;
            const float* xsl = reinterpret_cast<const float*>(ring + (size_t)s * kSlot + kWB) + sl * 4;
#pragma unroll 4
            for (int pc = 0; pc < KCE / 32; pc++) {
              const uint32_t wv = *reinterpret_cast<const uint32_t*>(wbase + pc * 128);
              uint64_t w01, w23;
              decode_pairs<WK>(wv, w01, w23);
#pragma unroll
              for (int b = 0; b < NB; b++) {
                const ulonglong2 xv =
                    *reinterpret_cast<const ulonglong2*>(xsl + b * KCE + pc * 32);
                fma2(acc01[b], w01, xv.x);
                fma2(acc23[b], w23, xv.y);
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
          // combine lanes: (g0+g1)+(g2+g3) per 8-lane position, then hsum8
          float v[4] = {lo_f(acc01[b]), hi_f(acc01[b]), lo_f(acc23[b]), hi_f(acc23[b])};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const float t1 = __fadd_rn(v[k], __shfl_xor_sync(0xffffffffu, v[k], 2));
            v[k] = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 4));
          }
#pragma unroll
          for (int k = 0; k < 4; k++) v[k] = __fadd_rn(v[k], __shfl_xor_sync(0xffffffffu, v[k], 1));
          float sum = __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
          const int gr = (gq0 + wc) * 4 + rq;
          const bool valid = ok && wc < gn && gr < ph.N;
          if (valid) sum = __fmul_rn(sum, ph.scale[gr]);
          float* y = ph.y + (long)b * ph.y_stride;
          if (ph.epi == EPI_SWIGLU) {
            const float up = __shfl_down_sync(0xffffffffu, sum, 8);
            if (valid && sl == 0 && (rq & 1) == 0) {
              const int o = gr >> 1;
              float sig;
              if (o < ph.silu_vec_limit)
                sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf_vec(__fsub_rn(0.0f, sum))));
              else
                sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf(-sum)));
              y[o] = __fmul_rn(__fmul_rn(sum, sig), up);
            }
          } else if (ph.epi == EPI_RESID) {
            if (valid && sl == 0) y[gr] = __fadd_rn(y[gr], sum);
          } else {
            if (valid && sl == 0) y[gr] = sum;
          }
        }
      }
    }
    // ---- phase done on this CTA: publish (release) for every other CTA
    asm volatile("bar.sync 1, %0;" ::"r"(nc));
    if (ct == 0) {
      fence_proxy_async();
      __threadfence();
      atomicAdd(P.ctr + p, 1);
    }
  }
  if (ct == 0) {
    __threadfence();
    if (atomicAdd(P.ctr + kMaxChainPhases, 1) == G - 1) {
      for (int p = 0; p <= kMaxChainPhases; p++) atomicExch(P.ctr + p, 0);
    }
  }
}

template <int WK, int NB>
cudaError_t launch_nb(const ChainParams& P, int grid, int smem, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(32 + 32 * kWarps);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_chain_nb_kernel<WK, NB>, P);
}

template <int WK>
cudaError_t dispatch_nb(int nb, const ChainParams& P, int grid, int smem, cudaStream_t s, bool pdl,
                        bool attr_only) {
  auto go = [&](auto kern, auto launch) -> cudaError_t {
    if (attr_only)
      return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - 256);
    return launch(P, grid, smem, s, pdl);
  };
  switch (nb) {
    case 2: return go(gemv_chain_nb_kernel<WK, 2>, launch_nb<WK, 2>);
    case 3: return go(gemv_chain_nb_kernel<WK, 3>, launch_nb<WK, 3>);
    case 4: return go(gemv_chain_nb_kernel<WK, 4>, launch_nb<WK, 4>);
    case 5: return go(gemv_chain_nb_kernel<WK, 5>, launch_nb<WK, 5>);
    case 6: return go(gemv_chain_nb_kernel<WK, 6>, launch_nb<WK, 6>);
    case 7: return go(gemv_chain_nb_kernel<WK, 7>, launch_nb<WK, 7>);
    case 8: return go(gemv_chain_nb_kernel<WK, 8>, launch_nb<WK, 8>);
  }
  return cudaErrorInvalidValue;
}

template <int WK, int KCE>
cudaError_t launch_t(const ChainParams& P, int grid, int smem, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(32 + 32 * kWarps);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_chain_kernel<WK, KCE>, P);
}

}  // namespace

int chain_kce(const ChainParams& P) {
  int kce = 0;
  for (int p = 0; p < P.nph; p++) {
    const int k = packed_kce(P.ph[p].K);
    if (kce && k != kce) return 0;
    kce = k;
  }
  return kce;
}

cudaError_t chain_prepare() {
  const int big = 227 * 1024 - 256;
  cudaError_t e = cudaFuncSetAttribute(gemv_chain_kernel<EC_W_INT8, 512>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (!e) e = cudaFuncSetAttribute(gemv_chain_kernel<EC_W_INT8, 32>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (!e) e = cudaFuncSetAttribute(gemv_chain_kernel<EC_W_FP8, 512>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  if (!e) e = cudaFuncSetAttribute(gemv_chain_kernel<EC_W_FP8, 32>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  ChainParams P{};
  for (int nb = 2; nb <= 8 && !e; nb++) {
    e = dispatch_nb<EC_W_INT8>(nb, P, 0, 0, nullptr, false, true);
    if (!e) e = dispatch_nb<EC_W_FP8>(nb, P, 0, 0, nullptr, false, true);
  }
  return e;
}

int chain_nb_smem(int kmax, int nb, int* stages) {
  const int fixed = 512 + ((kmax * 4 + 127) & ~127);
  const int slot = kWarps * 4 * 512 + nb * 512 * 4;
  int s = (227 * 1024 - 256 - fixed) / slot;
  if (s > kStagesMax) s = kStagesMax;
  if (s < 2) return -1;
  *stages = s;
  return fixed + s * slot;
}

cudaError_t chain_launch_nb(int wkind, ChainParams P, int nb, int grid, cudaStream_t s, bool pdl) {
  if (nb < 2 || nb > 8 || P.nph < 1 || P.nph > kMaxChainPhases) return cudaErrorInvalidValue;
  P.kmax = 0;
  for (int p = 0; p < P.nph; p++) {
    if (P.ph[p].pro != PRO_NORM_ROWS && (P.ph[p].K % 512)) return cudaErrorInvalidValue;
    if (P.ph[p].pro == PRO_NORM_ROWS && P.ph[p].K > P.kmax) P.kmax = P.ph[p].K;
  }
  int stages = 0;
  const int smem = chain_nb_smem(P.kmax, nb, &stages);
  if (smem < 0) return cudaErrorInvalidValue;
  P.stages = stages;
  if (wkind == EC_W_INT8) return dispatch_nb<EC_W_INT8>(nb, P, grid, smem, s, pdl, false);
  if (wkind == EC_W_FP8) return dispatch_nb<EC_W_FP8>(nb, P, grid, smem, s, pdl, false);
  return cudaErrorInvalidValue;
}

int chain_smem(const ChainParams& P, int kce, int* stages) {
  const int fixed = (2 * kStagesMax + 2) * 8 + 16 * 4 + P.kmax * 4 + ((P.knorm * 2 + 15) & ~15);
  const int sb = kWarps * 4 * kce;
  int s = (227 * 1024 - 256 - fixed) / sb;
  if (s > kStagesMax) s = kStagesMax;
  if (s < 2) return -1;
  *stages = s;
  return fixed + s * sb;
}

int chain_blocks_per_sm(int wkind, int kce, int kmax, int knorm) {
  ChainParams P{};
  P.kmax = kmax;
  P.knorm = knorm;
  int stages = 0;
  const int smem = chain_smem(P, kce, &stages);
  if (smem < 0) return 0;
  int n = 0;
  cudaError_t e = cudaErrorInvalidValue;
  const int threads = 32 + 32 * kWarps;
  if (wkind == EC_W_INT8)
    e = kce == 512 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                         &n, gemv_chain_kernel<EC_W_INT8, 512>, threads, smem)
                   : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                         &n, gemv_chain_kernel<EC_W_INT8, 32>, threads, smem);
  else if (wkind == EC_W_FP8)
    e = kce == 512 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                         &n, gemv_chain_kernel<EC_W_FP8, 512>, threads, smem)
                   : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                         &n, gemv_chain_kernel<EC_W_FP8, 32>, threads, smem);
  return e == cudaSuccess ? n : 0;
}

cudaError_t chain_launch(int wkind, ChainParams P, int grid, cudaStream_t s, bool pdl) {
  const int kce = chain_kce(P);
  if (!kce || P.nph < 1 || P.nph > kMaxChainPhases) return cudaErrorInvalidValue;
  P.kmax = 0;
  P.knorm = 0;
  for (int p = 0; p < P.nph; p++) {
    P.kmax = P.ph[p].K > P.kmax ? P.ph[p].K : P.kmax;
    if (P.ph[p].pro == PRO_RMSNORM && P.ph[p].K > P.knorm) P.knorm = P.ph[p].K;
  }
  int stages = 0;
  const int smem = chain_smem(P, kce, &stages);
  if (smem < 0) return cudaErrorInvalidValue;
  P.stages = stages;
  if (wkind == EC_W_INT8)
    return kce == 512 ? launch_t<EC_W_INT8, 512>(P, grid, smem, s, pdl)
                      : launch_t<EC_W_INT8, 32>(P, grid, smem, s, pdl);
  if (wkind == EC_W_FP8)
    return kce == 512 ? launch_t<EC_W_FP8, 512>(P, grid, smem, s, pdl)
                      : launch_t<EC_W_FP8, 32>(P, grid, smem, s, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace ec

#ifdef EC_PHASE_TIMING
extern "C" int ec_debug_chain_times(long long* out) {
  return cudaMemcpyFromSymbol(out, ec::g_chain_ts, 64 * sizeof(long long)) == cudaSuccess ? 0 : -2;
}
#endif
