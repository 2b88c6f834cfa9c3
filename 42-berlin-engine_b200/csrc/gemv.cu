// gemv.cu -- batch-1 GEMV that streams the weight matrix from HBM once, at
// bandwidth, and reproduces the reference's floating-point result bit for bit.
//
// Reference order (matvec_bf16_f32_blocked, src/compute/ops_matmul.c:57-141):
// each row is summed in 32 lanes; lane L owns elements j == L (mod 32) and
// accumulates them with one FMA each, in increasing j; the four 8-lane groups
// combine as (g0+g1)+(g2+g3); an 8-lane horizontal sum gives the row.
//
// B200 mapping:
//   * one CTA per SM takes a contiguous, balanced range of rows;
//   * warp 0 is a producer: one lane streams row segments of `kcb` bytes with
//     1-D bulk copies (cp.async.bulk) into a 4-stage shared-memory ring,
//     completing on mbarriers; it needs nothing from the previous kernel, so
//     under programmatic dependent launch it starts while that kernel drains;
//   * 8 consumer threads per row, thread s owning lanes 4s..4s+3 for the whole
//     row, so every lane's FMA chain runs in the reference's order in one
//     thread; each thread reads 4 weight bytes and one float4 of x per 32
//     elements (row stride padded by 32 bytes: conflict-free);
//   * lane combination with three xor-shuffles in the reference's order;
//   * optional prologue: the RMSNorm of x in the reference's order
//     (rmsnorm_f32_avx2, ops_norm.c:27-124), overlapping the first stages;
//   * epilogues: store, residual add (simd_add_f32: x + y), or SwiGLU on
//     interleaved gate/up rows (op_silu_mul_fused_f32, ops_activation.c:48).
#include "ec_internal.cuh"
#include "gemv.cuh"

namespace ec {

constexpr int kStages = 4;
constexpr int kRowPad = 32;
constexpr int kMaxRg = 32;

template <int WK>
struct WTraits;
template <>
struct WTraits<EC_W_INT8> {
  static constexpr int esize = 1;
};
template <>
struct WTraits<EC_W_FP8> {
  static constexpr int esize = 1;
};
template <>
struct WTraits<EC_W_BF16> {
  static constexpr int esize = 2;
};

template <int WK>
__device__ __forceinline__ void decode4(const uint8_t* p, float* f) {
  if constexpr (WK == EC_W_INT8) {
    dec_i8x4(*reinterpret_cast<const uint32_t*>(p), f);
  } else if constexpr (WK == EC_W_FP8) {
    dec_fp8x4(*reinterpret_cast<const uint32_t*>(p), f);
  } else {
    uint2 u = *reinterpret_cast<const uint2*>(p);
    dec_bf16x2(u.x, f);
    dec_bf16x2(u.y, f + 2);
  }
}

template <int WK, int PRO, int EPI>
__global__ void __launch_bounds__(32 + 8 * kMaxRg, 1) gemv_kernel(GemvParams p) {
  constexpr int ES = WTraits<WK>::esize;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStages;
  uint64_t* xbar = empty + kStages;                         // x arrival (+ 1 pad)
  float* red = reinterpret_cast<float*>(xbar + 2);          // 16 floats
  float* xs = red + 16;                                     // [K]
  uint8_t* stages = reinterpret_cast<uint8_t*>(xs + p.K);
  const int kcb = p.kcb;
  const int rstride = kcb + kRowPad;
  const int stage_bytes = p.rg * rstride;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nc = blockDim.x - 32;  // consumer threads
  const int ncw = nc >> 5;         // consumer warps

  constexpr int U = (EPI == EPI_SWIGLU) ? 2 : 1;
  const long nu = p.N / U;
  const int r0 = (int)(nu * blockIdx.x / gridDim.x) * U;
  const int r1 = (int)(nu * (blockIdx.x + 1) / gridDim.x) * U;
  const int nrows = r1 - r0;
  const int ngroups = (nrows + p.rg - 1) / p.rg;
  const long kbytes = (long)p.K * ES;
  const int nchunks = (int)(kbytes / kcb);
  const int ntasks = ngroups * nchunks;

  if (tid == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ncw);
    }
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int t = 0; t < ntasks; t++) {
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(&empty[s], ((t / kStages) - 1) & 1, p.err)) return;
        const int g = t / nchunks;
        const int c = t - g * nchunks;
        const int gr0 = r0 + g * p.rg;
        const int gn = min(p.rg, r1 - gr0);
        mbar_expect_tx(&full[s], (uint32_t)(gn * kcb));
        uint8_t* dst = stages + s * stage_bytes;
        const uint8_t* src = p.w + (long)gr0 * kbytes + (long)c * kcb;
        for (int r = 0; r < gn; r++) bulk_g2s(dst + r * rstride, src + (long)r * kbytes, kcb, &full[s]);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int ct = tid - 32;
  pdl_wait();
  if (ct == 0) {
    // x (written by the previous kernel) arrives with one bulk copy
    mbar_expect_tx(xbar, (uint32_t)(p.K * 4));
    bulk_g2s(xs, p.x, (uint32_t)(p.K * 4), xbar);
  }
  bool ok = mbar_wait(xbar, 0, p.err);
  if constexpr (PRO == PRO_RMSNORM) rmsnorm_smem(xs, p.norm_w, p.K, p.eps, red, ct, nc);

  const int r = ct >> 3;   // row within group
  const int sl = ct & 7;   // lane quad: lanes 4*sl .. 4*sl+3
  const int kce = kcb / ES;  // elements per chunk
  float acc[4];

  for (int t = 0; t < ntasks; t++) {
    const int s = t % kStages;
    const int g = t / nchunks;
    const int c = t - g * nchunks;
    if (c == 0) {
#pragma unroll
      for (int i = 0; i < 4; i++) acc[i] = 0.0f;
    }
    if (ok) ok = mbar_wait(&full[s], (t / kStages) & 1, p.err);
    if (ok) {
      const uint8_t* row = stages + s * stage_bytes + r * rstride + sl * 4 * ES;
      const float* xc = xs + c * kce + sl * 4;
#pragma unroll 8
      for (int j = 0; j < kce; j += 32) {
        float wv[4];
        decode4<WK>(row + j * ES, wv);
        const float4 xv = *reinterpret_cast<const float4*>(xc + j);
        acc[0] = __fmaf_rn(wv[0], xv.x, acc[0]);
        acc[1] = __fmaf_rn(wv[1], xv.y, acc[1]);
        acc[2] = __fmaf_rn(wv[2], xv.z, acc[2]);
        acc[3] = __fmaf_rn(wv[3], xv.w, acc[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    if (c == nchunks - 1) {
      // combine lanes: (g0+g1)+(g2+g3) per 8-lane position, then hsum8
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float t1 = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 2));
        v[i] = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 4));
      }
#pragma unroll
      for (int i = 0; i < 4; i++) v[i] = __fadd_rn(v[i], __shfl_xor_sync(0xffffffffu, v[i], 1));
      float sum = __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
      const int gr = r0 + g * p.rg + r;
      const bool valid = ok && (r < p.rg) && (gr < r1);
      if constexpr (WK != EC_W_BF16) {
        if (valid) sum = __fmul_rn(sum, p.scale[(long)gr * p.scale_stride]);
      }
      if constexpr (EPI == EPI_SWIGLU) {
        const float up = __shfl_down_sync(0xffffffffu, sum, 8);
        if (valid && sl == 0 && (r & 1) == 0) {
          const int i = gr >> 1;
          float sig;
          if (i < p.silu_vec_limit)
            sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf_vec(__fsub_rn(0.0f, sum))));
          else
            sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_expf(-sum)));
          p.y[i] = __fmul_rn(__fmul_rn(sum, sig), up);
        }
      } else if constexpr (EPI == EPI_RESID) {
        if (valid && sl == 0) p.y[gr] = __fadd_rn(p.y[gr], sum);
      } else {
        if (valid && sl == 0) p.y[gr] = sum;
      }
    }
  }
}

static int pick_kcb(long kbytes, int es) {
  // largest divisor of kbytes that is a multiple of 32 elements and 16 bytes,
  // at most 2048 bytes
  const int unit = 32 * es;
  for (int c = 2048; c >= unit; c -= unit)
    if (kbytes % c == 0 && c % 16 == 0) return c;
  return 0;
}

bool gemv_plan(int wkind, int N, int K, int epi, int n_sm, GemvPlan* plan) {
  const int es = (wkind == EC_W_BF16) ? 2 : 1;
  if (N <= 0 || K <= 0 || K % 32 != 0) return false;
  if (epi == EPI_SWIGLU && (N % 2) != 0) return false;
  const long kbytes = (long)K * es;
  int kcb = pick_kcb(kbytes, es);
  if (!kcb) return false;
  const int unit = (epi == EPI_SWIGLU) ? 2 : 1;
  int grid = n_sm;
  if (N / unit < grid) grid = N / unit;
  const int rows_max = ((N / unit + grid - 1) / grid) * unit;
  const int ngroups = (rows_max + kMaxRg - 1) / kMaxRg;
  int rg = (rows_max + ngroups - 1) / ngroups;
  rg = (rg + 3) & ~3;  // whole warps of 4 rows (SwiGLU pairs stay in a warp)
  if (rg > kMaxRg) rg = kMaxRg;
  // shrink the chunk when the ring would not fit next to x
  int smem;
  for (;;) {
    smem = (2 * kStages + 2) * 8 + 16 * 4 + K * 4 + kStages * rg * (kcb + kRowPad);
    if (smem <= 220 * 1024) break;
    int c2 = kcb / 2;
    if (c2 < 32 * es || kbytes % c2 != 0 || c2 % 16 != 0) return false;
    kcb = c2;
  }
  plan->grid = grid;
  plan->block = 32 + 8 * rg;
  plan->smem = smem;
  plan->rg = rg;
  plan->kcb = kcb;
  return true;
}

template <int WK, int PRO, int EPI>
static cudaError_t set_attr() {
  return cudaFuncSetAttribute(gemv_kernel<WK, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              220 * 1024);
}

template <int WK>
static cudaError_t set_attr_w() {
  cudaError_t e = cudaSuccess;
  if (!e) e = set_attr<WK, PRO_NONE, EPI_STORE>();
  if (!e) e = set_attr<WK, PRO_NONE, EPI_RESID>();
  if (!e) e = set_attr<WK, PRO_NONE, EPI_SWIGLU>();
  if (!e) e = set_attr<WK, PRO_RMSNORM, EPI_STORE>();
  if (!e) e = set_attr<WK, PRO_RMSNORM, EPI_RESID>();
  if (!e) e = set_attr<WK, PRO_RMSNORM, EPI_SWIGLU>();
  return e;
}

// Opt every instantiation into large dynamic shared memory on the current
// device (outside any stream capture).
cudaError_t gemv_prepare() {
  cudaError_t e = set_attr_w<EC_W_INT8>();
  if (!e) e = set_attr_w<EC_W_FP8>();
  if (!e) e = set_attr_w<EC_W_BF16>();
  return e;
}

template <int WK, int PRO, int EPI>
static cudaError_t launch_t(const GemvPlan& plan, const GemvParams& p, cudaStream_t stream,
                            bool pdl) {
  auto fn = gemv_kernel<WK, PRO, EPI>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(plan.block);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  GemvParams q = p;
  q.rg = plan.rg;
  q.kcb = plan.kcb;
  return cudaLaunchKernelEx(&cfg, fn, q);
}

template <int WK>
static cudaError_t launch_w(int pro, int epi, const GemvPlan& plan, const GemvParams& p,
                            cudaStream_t s, bool pdl) {
  if (pro == PRO_RMSNORM) {
    if (epi == EPI_SWIGLU) return launch_t<WK, PRO_RMSNORM, EPI_SWIGLU>(plan, p, s, pdl);
    if (epi == EPI_RESID) return launch_t<WK, PRO_RMSNORM, EPI_RESID>(plan, p, s, pdl);
    return launch_t<WK, PRO_RMSNORM, EPI_STORE>(plan, p, s, pdl);
  }
  if (epi == EPI_SWIGLU) return launch_t<WK, PRO_NONE, EPI_SWIGLU>(plan, p, s, pdl);
  if (epi == EPI_RESID) return launch_t<WK, PRO_NONE, EPI_RESID>(plan, p, s, pdl);
  return launch_t<WK, PRO_NONE, EPI_STORE>(plan, p, s, pdl);
}

cudaError_t gemv_launch(int wkind, int pro, int epi, const GemvPlan& plan, const GemvParams& p,
                        cudaStream_t stream, bool pdl) {
  if (wkind == EC_W_INT8) return launch_w<EC_W_INT8>(pro, epi, plan, p, stream, pdl);
  if (wkind == EC_W_FP8) return launch_w<EC_W_FP8>(pro, epi, plan, p, stream, pdl);
  return launch_w<EC_W_BF16>(pro, epi, plan, p, stream, pdl);
}

}  // namespace ec
