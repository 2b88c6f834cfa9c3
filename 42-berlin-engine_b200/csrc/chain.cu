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
  uint8_t* stages = reinterpret_cast<uint8_t*>(xs + P.kmax);
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
  bool ok = true;
  int t = 0;
  for (int p = 0; p < P.nph; p++) {
    const ChainPhase& ph = P.ph[p];
    // ---- the input vector: complete once every CTA finished phase p-1
    if (p == 0) {
      pdl_wait();
    } else {
      if (ct == 0) {
        bool got = false;
        for (uint32_t it = 0; it < kWaitLimit && ok; it++)
          if (ld_acquire(P.ctr + p - 1) >= G) {
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
      mbar_expect_tx(xbar, (uint32_t)(ph.K * 4));
      bulk_g2s(xs, ph.x, (uint32_t)(ph.K * 4), xbar);
    }
    if (ok) ok = mbar_wait(xbar, p & 1, P.err);
    if (ph.pro == PRO_RMSNORM && ok) rmsnorm_smem(xs, ph.norm_w, ph.K, P.eps, red, ct, nc);

    // ---- this CTA's rows, group by group, slot by slot
    const Split sp = split(ph, blockIdx.x, G);
    for (int g = 0; g < sp.ngroups; g++) {
      const int gq0 = sp.q0 + g * sp.qs, gn = min(sp.qs, sp.q1 - gq0);
      uint64_t acc01 = 0, acc23 = 0;
      for (int c0 = 0; c0 < sp.nchunks; c0 += sp.m, t++) {
        const int s = t % S, mc = min(sp.m, sp.nchunks - c0);
        if (ok) ok = mbar_wait(&full[s], (t / S) & 1, P.err);
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
  return e;
}

int chain_smem(const ChainParams& P, int kce, int* stages) {
  const int fixed = (2 * kStagesMax + 2) * 8 + 16 * 4 + P.kmax * 4;
  const int sb = kWarps * 4 * kce;
  int s = (227 * 1024 - 256 - fixed) / sb;
  if (s > kStagesMax) s = kStagesMax;
  if (s < 2) return -1;
  *stages = s;
  return fixed + s * sb;
}

cudaError_t chain_launch(int wkind, ChainParams P, int grid, cudaStream_t s, bool pdl) {
  const int kce = chain_kce(P);
  if (!kce || P.nph < 1 || P.nph > kMaxChainPhases) return cudaErrorInvalidValue;
  P.kmax = 0;
  for (int p = 0; p < P.nph; p++) P.kmax = P.ph[p].K > P.kmax ? P.ph[p].K : P.kmax;
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
